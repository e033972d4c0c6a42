"""The C ABI library: loads without a GPU, exports every entry point include/smlm_b200.h declares, rejects bad
arguments on the host (no launch), and the Python layer refuses CPU tensors (there is no CPU fallback)."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT
from smlm_b200 import _lib as L
from smlm_b200 import kernels as K

HEADER = os.path.join(ROOT, "include", "smlm_b200.h")


def declared():
    text = open(HEADER).read()
    return re.findall(r"SMLM_API\s+[\w\s\*]*?\b(smlm_\w+)\s*\(", text)


def test_library_exports_every_declared_entry_point():
    names = declared()
    assert len(names) >= 14
    so = ctypes.CDLL(L.LIB_PATH)
    for n in names:
        assert hasattr(so, n), f"{n} declared in smlm_b200.h but not exported"
    assert set(names) == set(L.SIGNATURES), "ctypes signatures out of sync with the header"
    lib = L.load()
    assert lib.smlm_version() >= 100


def test_host_side_argument_checks_return_invalid():
    lib = L.load()
    s = ctypes.c_void_p(0x1000)   # never dereferenced: the checks fail before any launch
    rc = lib.smlm_pk_select(s, s, L.BF16, 4, 2, 64, 33, s, s, s, None)
    assert rc == L.ERR_INVALID and b"knn" in lib.smlm_last_error()
    rc = lib.smlm_pk_select(s, s, L.BF16, 4, 2, 1 << 17, 32, s, s, s, None)
    assert rc == L.ERR_INVALID
    rc = lib.smlm_bag_forward(s, s, L.F32, s, 7, 4, 8, 16, 32, s, L.F32, None, None)
    assert rc == L.ERR_INVALID and b"table" in lib.smlm_last_error()
    rc = lib.smlm_rowwise_step(s, s, s, s, None, None, 1.0, 10, 8, L.ROWRMS, 0.95, 1e-8, 0.01, 0, s, 0, None)
    assert rc == L.ERR_INVALID and b"count" in lib.smlm_last_error()
    rc = lib.smlm_quantize_q4(s, 10, 7, s, s, None)
    assert rc == L.ERR_INVALID
    rc = lib.smlm_lazy_adam_step(s, s, s, s, s, None, 1.0, 10, 8, 0.1, 0.9, 0.1, 1.0, 1e-8, -1e-3, None, 0, 8, s, 0,
                                 None)
    assert rc == L.ERR_INVALID and b"flags" in lib.smlm_last_error()
    assert rc == L.ERR_INVALID
    # the allocation-free scoring refuses calls beyond its static scratch without forming n * heads (2^62 x 4
    # would wrap to 0)
    for n in (1 << 62, 16384 // 4 + 1):
        rc = lib.smlm_score_select_noalloc(s, s, n, 4, 1024, 128, 32, s, s, s, None, None)
        assert rc == L.ERR_INVALID and b"SMLM_NOALLOC_MAX_ROWS" in lib.smlm_last_error()
    with pytest.raises(ValueError, match="knn"):
        L.check(lib.smlm_pk_select(s, s, L.BF16, 4, 2, 64, 0, s, s, s, None), "pk_select")
    # empty inputs are fine and launch nothing
    assert lib.smlm_bag_forward(None, None, L.F32, None, L.F32, 0, 8, 16, 32, None, L.F32, None, None) == L.OK


def test_python_api_refuses_cpu_tensors():
    t = torch.zeros(16, 8)
    idx = torch.zeros(2, 4, dtype=torch.long)
    w = torch.zeros(2, 4)
    with pytest.raises(ValueError, match="CUDA"):
        K.bag_forward(idx, w, t)
    with pytest.raises(ValueError, match="CUDA"):
        K.pk_select(torch.zeros(2, 2, 16, dtype=torch.bfloat16), torch.zeros(2, 2, 16, dtype=torch.bfloat16), 4)
    from smlm_b200.pkm import ProductKeyMemory
    mem = ProductKeyMemory(16, 16, n_keys=8, heads=2, knn=4, k_dim=8, query_norm="none", swilu=False)
    with pytest.raises(ValueError, match="CUDA"):
        mem(torch.zeros(3, 16))
    from smlm_b200.sparse_values import LazyRowAdam
    with pytest.raises(ValueError, match="CUDA"):
        LazyRowAdam([torch.nn.Parameter(torch.zeros(16, 8))], lr=1e-3)


def test_layer_rejects_unsupported_shapes():
    from smlm_b200.pkm import ProductKeyMemory
    with pytest.raises(ValueError, match="knn"):
        ProductKeyMemory(32, 32, n_keys=64, knn=33, k_dim=16)
    with pytest.raises(ValueError, match="n_keys"):
        ProductKeyMemory(32, 32, n_keys=1 << 17, knn=4, k_dim=16)
    # any n_keys / knn within the limits, powers of two or not (the reference's Triton path needed powers of two)
    ProductKeyMemory(32, 32, n_keys=24, knn=5, k_dim=16)


def test_state_dict_formats_match_reference():
    from smlm_b200.pkm import ProductKeyMemory
    mem = ProductKeyMemory(24, 24, n_keys=16, heads=2, knn=4, k_dim=16)
    keys = set(mem.state_dict())
    assert {"keys", "query_proj.weight", "query_proj.bias", "values.weight", "swilu_proj.weight",
            "value_proj.weight", "query_norm.running_mean"} <= keys
    from smlm_b200.row_optim import state_bytes
    assert state_bytes("rowrms", 100) == 804 and state_bytes("rowadagrad", 100) == 404


@pytest.mark.parametrize("mode", ["fp32", "bf16", "int8"])
def test_lazy_adam_argument_validation(mode):
    """The reference's constructor checks (tests/test_lowmem_values.py), before any device work."""
    from smlm_b200.sparse_values import LazyRowAdam
    P = torch.nn.Parameter
    for dtype in (torch.float16, torch.bfloat16, torch.float64):
        with pytest.raises(ValueError, match="fp32|float32"):
            LazyRowAdam([P(torch.zeros(4, 7, dtype=dtype))], lr=0.01, state_dtype=mode)
    for shape in ((5,), (2, 3, 4), (2, 0)):
        with pytest.raises(ValueError, match="contiguous fp32 tables"):
            LazyRowAdam([P(torch.zeros(shape))], lr=0.01, state_dtype=mode)
    with pytest.raises(ValueError, match="contiguous fp32 tables"):
        LazyRowAdam([P(torch.zeros(7, 11).t())], lr=0.01, state_dtype=mode)
    for options in ({"lr": float("nan")}, {"eps": float("nan")}, {"lr": -0.1}, {"eps": -0.1}, {"betas": (0.9, 1.0)}):
        with pytest.raises(ValueError):
            LazyRowAdam([P(torch.zeros(4, 7))], state_dtype=mode, **dict({"lr": 0.01}, **options))
    with pytest.raises(ValueError, match="state_dtype"):
        LazyRowAdam([P(torch.zeros(4, 7))], lr=0.01, state_dtype="fp16")


def test_nvtx_ranges_balanced(monkeypatch):
    """SMLM_B200_NVTX: every library call opens one NVTX range named after it and closes it, also on an error."""
    from smlm_b200 import _lib as L
    log = []
    monkeypatch.setattr(L, "NVTX", True)
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: log.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: log.append(("pop",)))
    with L.timed("bag_forward", 1):
        pass
    with pytest.raises(ValueError):
        with L.timed("lazy_adam_step", 2):
            raise ValueError("argument check")
    assert log == [("push", "smlm:bag_forward"), ("pop",), ("push", "smlm:lazy_adam_step"), ("pop",)]
    monkeypatch.setattr(L, "NVTX", False)
    with L.timed("bag_forward", 1):
        pass
    assert len(log) == 4


def test_reference_named_lowmem_step_validates_before_launch():
    """kernels.lazy_adam_step_lowmem (the reference's signature) refuses a bad state_dtype, missing int8 scales,
    mismatched moment dtypes and CPU tensors with ValueError, before any launch."""
    p = torch.zeros(4, 8)
    acc, touched = torch.zeros(4, 8), torch.zeros(4, dtype=torch.bool)
    bf = torch.zeros(4, 8, dtype=torch.bfloat16)
    args = (acc, touched, 1.0, 1, 1e-3, 0.9, 0.98, 1e-8)
    with pytest.raises(ValueError, match="'bf16' or 'int8'"):
        K.lazy_adam_step_lowmem(p, bf, bf, *args, "fp16")
    with pytest.raises(ValueError, match="scale"):
        K.lazy_adam_step_lowmem(p, torch.zeros(4, 8, dtype=torch.int8), torch.zeros(4, 8, dtype=torch.uint8),
                                *args, "int8")
    with pytest.raises(ValueError, match="needs moments"):
        K.lazy_adam_step_lowmem(p, bf, bf, *args, "int8", torch.zeros(4), torch.zeros(4))
    with pytest.raises(ValueError, match="CUDA"):
        K.lazy_adam_step_lowmem(p, bf, bf, *args, "bf16")


def test_reference_launch_arguments_accepted():
    """The reference's Triton launch-shape arguments are accepted by name (no TypeError); the call then reaches the
    usual argument checks (CPU tensors: ValueError, no CPU path)."""
    t = torch.zeros(4, 8)
    idx = torch.zeros(2, 3, dtype=torch.int64)
    w = torch.zeros(2, 3)
    s = torch.zeros(2, 4, 16)
    calls = [
        lambda: K.pk_select(s, s, 4, ch=128, num_warps=4),
        lambda: K.bag_forward(idx, w, t, block_j=32, block_d=128),
        lambda: K.bag_infer(idx, w, t, block_j=64, block_d=None),
        lambda: K.bag_backward_rows(torch.zeros(2, 8), idx, w, t, torch.zeros(4, 8),
                                    torch.zeros(4, dtype=torch.bool), P=32, block_d=64, num_warps=2),
        lambda: K.lazy_adam_step(t, t, t, t, torch.zeros(4, dtype=torch.bool), 1.0, 1, 1e-3, 0.9, 0.98, 1e-8,
                                 rows_per_program=8, block_d=128),
    ]
    for call in calls:
        with pytest.raises(ValueError):
            call()


def test_header_compiles_as_c_and_links(tmp_path):
    """The header is plain C11 (gcc -std=c11 -pedantic -Werror), every declaration links by name against
    libsmlm_b200.so, and a C caller gets the size queries, the host-side argument checks and the error text
    without a GPU (no call below reaches a launch)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    names = declared()
    src = tmp_path / "abi_caller.c"
    src.write_text("\n".join([
        "#include <stdio.h>",
        "#include <string.h>",
        '#include "smlm_b200.h"',
        "typedef void (*fn_t)(void);",
        "static const fn_t every_entry_point[] = {" + ", ".join(f"(fn_t){n}" for n in names) + "};",
        "int main(void) {",
        "    void *s = (void *)0x1000; /* never dereferenced: the checks fail before any launch */",
        "    if (smlm_version() < 100) return 1;",
        "    if (smlm_bag_backward_workspace(1024, 128, 1 << 20, 384) == 0) return 2;",
        "    if (smlm_touched_workspace(1 << 20) == 0) return 3;",
        "    if (smlm_pk_select(s, s, SMLM_BF16, 4, 2, 64, 33, s, s, s, NULL) != SMLM_ERR_INVALID) return 4;",
        '    if (strstr(smlm_last_error(), "knn") == NULL) return 5;',
        "    if (smlm_bag_forward(NULL, NULL, SMLM_F32, NULL, SMLM_F32, 0, 8, 16, 32, NULL, SMLM_F32, NULL, NULL)",
        "        != SMLM_OK) return 6;",
        '    printf("ok %zu\\n", sizeof(every_entry_point) / sizeof(every_entry_point[0]));',
        "    return 0;",
        "}",
    ]) + "\n")
    lib_dir = os.path.dirname(L.LIB_PATH)
    exe = tmp_path / "abi_caller"
    subprocess.run([gcc, "-std=c11", "-pedantic", "-Wall", "-Wextra", "-Werror", "-I", os.path.dirname(HEADER),
                    str(src), "-o", str(exe), "-L", lib_dir, "-lsmlm_b200", f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.strip() == f"ok {len(names)}"


def test_every_declaration_cites_its_reference_interface():
    """Each entry point of the header names the reference interface it replaces (file:line) or says that it has no
    counterpart there: in the comment above it, above its group of adjacent declarations, or in its section's
    heading comment."""
    text = open(HEADER).read()
    cite = re.compile(r"\.(py|c):\d+|[Nn]o counterpart")
    uncited = []
    for sec in re.split(r"/\* -{10,}", text):
        heading = re.match(r"[^\n]*\n?((?: \*[^\n]*\n)*)", sec).group(0)
        covered = bool(cite.search(heading))
        prev, prev_ok = 0, False
        for m in re.finditer(r"SMLM_API\s+[\w\s\*]*?\b(smlm_\w+)\s*\(", sec):
            between = sec[prev:m.start()]
            ok = covered or bool(cite.search(between)) or (prev > 0 and not between.strip() and prev_ok)
            if not ok:
                uncited.append(m.group(1))
            prev, prev_ok = sec.index(";", m.end()) + 1, ok
    assert not uncited, f"declarations without a reference citation: {uncited}"
