"""Loads libsmlm_b200.so (the sm_100a kernels behind include/smlm_b200.h) and wraps its C ABI for PyTorch tensors.

There is no fallback: if the library is missing or a tensor is not on a CUDA device, the call raises. Tensors
stay owned by PyTorch (caching allocator); every call passes raw device pointers plus the current CUDA stream,
and scratch memory is a torch uint8 buffer sized by the library's own *_workspace query.

SMLM_B200_CHECK=1 turns on checked mode: after every call the stream is synchronised and the device status
word (out-of-range row indices) is read; a set flag raises IndexError.

SMLM_B200_NVTX=1 wraps every library call in an NVTX range named "smlm:<call>" (score_select, bag_forward,
bag_backward_rows, lazy_adam_step, xchg_forward, ...), so a profiler timeline shows the layer's stages; off by
default (a range costs host time on every call).
"""
import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libsmlm_b200.so")

OK, ERR_INVALID, ERR_CUDA, ERR_WORKSPACE = 0, 1, 2, 3
F32, BF16, F16, Q4 = 0, 1, 2, 3
I32, I64, I8 = 4, 5, 6
FLAG_INDEX_RANGE = 1
FLAG_TIMEOUT = 4
ROWRMS, ROWADAGRAD = 0, 1
BWD_FIRST_TOUCH_WRITES = 1
BWD_DEFER_ROWS = 2
STEP_KEEP_ACC = 1
ROWS_TO_CURRENT = 1
SCORE_F32_EXACT, SCORE_BF16 = 0, 1

# Kernel launches behind one call, for the benchmark's launch count (checked against the ncu launch list):
# the backward = key build + radix sort (histogram, exclusive sum, one onesweep pass per 8 key bits at the
# benchmark's 25-bit rows) + segment pass + fix-up; touched-row compaction = cub select (tile-state init + scan).
COMPACT_LAUNCHES = 2


def backward_launches(rows):
    """Launches of one smlm_bag_backward_rows call over a table of `rows` rows (sort keys carry rows + 1 values)."""
    bits = max(1, int(rows).bit_length())
    return 1 + 2 + (bits + 7) // 8 + 2

_p, _i64, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/smlm_b200.h
SIGNATURES = {
    "smlm_version": (_i32, []),
    "smlm_last_error": (ctypes.c_char_p, []),
    "smlm_bag_forward": (_i32, [_p, _p, _i32, _p, _i32, _i64, _i64, _i64, _i64, _p, _i32, _p, _p]),
    "smlm_bag_infer": (_i32, [_p, _p, _i32, _p, _i32, _p, _p, _i32, _i64, _i64, _i64, _i64, _p, _i32, _p, _p]),
    "smlm_quantize_q4": (_i32, [_p, _i64, _i64, _p, _p, _p]),
    "smlm_bag_backward_workspace": (_sz, [_i64, _i64, _i64, _i64]),
    "smlm_bag_backward_rows": (_i32, [_p, _i32, _p, _p, _i32, _p, _i32, _p, _p, _p, _i32, _p, _i64, _i64, _i64,
                                      _i64, _p, _sz, _p, _p]),
    "smlm_touched_workspace": (_sz, [_i64]),
    "smlm_bag_rows_materialize": (_i32, [_p, _i32, _p, _i32, _p, _i64, _i64, _i64, _i64, _p, _sz, _p]),
    "smlm_lazy_adam_deferred_step": (_i32, [_p, _p, _p, _p, _p, _i32, _p, _i32, _p, _f32, _i64, _i64, _i64, _i64,
                                            _f32, _f32, _f32, _f32, _f32, _f32, _p, _i32, _p, _sz, _p]),
    "smlm_lazy_adam_deferred_step_dev": (_i32, [_p, _p, _p, _p, _p, _i32, _p, _i32, _p, _f32, _i64, _i64, _i64, _i64,
                                                _p, _p, _i32, _p, _sz, _p]),
    "smlm_lazy_adam_step": (_i32, [_p, _p, _p, _p, _p, _p, _f32, _i64, _i64, _f32, _f32, _f32, _f32, _f32, _f32,
                                   _p, _i32, _i32, _p, _sz, _p]),
    "smlm_lazy_adam_step_dev": (_i32, [_p, _p, _p, _p, _p, _p, _f32, _i64, _i64, _p, _p, _i32, _i32, _p, _sz, _p]),
    "smlm_lazy_adam_lowmem_step": (_i32, [_p, _p, _p, _p, _p, _i32, _p, _p, _p, _f32, _i64, _i64, _f32, _f32, _f32,
                                          _f32, _f32, _f32, _f32, _p, _i32, _i32, _p, _sz, _p]),
    "smlm_rowwise_step": (_i32, [_p, _p, _p, _p, _p, _p, _f32, _i64, _i64, _i32, _f32, _f32, _f32, _i32, _p, _sz,
                                 _p]),
    "smlm_rowwise_deferred_step": (_i32, [_p, _p, _p, _p, _p, _i32, _p, _i32, _p, _f32, _i64, _i64, _i64, _i64,
                                          _i32, _f32, _f32, _f32, _p, _sz, _p]),
    "smlm_touched_norm": (_i32, [_p, _p, _p, _i64, _i64, _p, _p, _sz, _p]),
    "smlm_zero_untouched": (_i32, [_p, _p, _i64, _i64, _p]),
    "smlm_pk_select": (_i32, [_p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "smlm_select_backward": (_i32, [_p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "smlm_select_grad_entries": (_i32, [_p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "smlm_subkey_scores_f32": (_i32, [_p, _p, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "smlm_score_select_workspace": (_sz, [_i64, _i64]),
    "smlm_score_select": (_i32, [_p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _sz, _p, _p]),
    "smlm_shard_bag_forward": (_i32, [_p, _i32, _i64, _p, _i32, _p, _i32, _i64, _i64, _i64, _i64, _p, _i32, _p]),
    "smlm_shard_bag_backward_rows": (_i32, [_p, _i32, _p, _i32, _i64, _p, _i32, _p, _i32, _p, _p, _p, _i32, _p,
                                            _i64, _i64, _i64, _i64, _p, _sz, _p, _p]),
    "smlm_slot_sum": (_i32, [_p, _i64, _i64, _p, _p]),
    "smlm_xchg_bytes": (_sz, [_i32, _i64, _i64, _i64]),
    "smlm_xchg_alloc": (_i32, [_sz, _p, _p]),
    "smlm_xchg_open": (_i32, [_p, _p]),
    "smlm_xchg_close": (_i32, [_p]),
    "smlm_xchg_free": (_i32, [_p]),
    "smlm_xchg_forward": (_i32, [_p, _p, _i32, _i32, _p, _p, _i64, _i64, _i64, _i64, _p, _i32, _i64, _i64, _i64,
                                 _p, _p, _p, _i32, _p, _i32, _i64, _p, _p]),
    "smlm_xchg_backward_gw": (_i32, [_p, _i32, _i32, _p, _i32, _p, _i64, _i64, _i64, _p, _i32, _i64, _i64, _i64,
                                     _i64, _p, _p]),
    "smlm_xchg_collect_gw": (_i32, [_p, _i32, _i32, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "smlm_score_select_noalloc": (_i32, [_p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p]),
    "smlm_ngram_rows": (_i32, [_p, _i64, _i64, _i32, _p, _p, _i32, _i32, _i32, _i64, _p, _p]),
    "smlm_host_register": (_i32, [_p, _sz, _p]),
    "smlm_host_unregister": (_i32, [_p]),
    "smlm_host_rows_gather": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _p]),
    "smlm_host_rows_scatter": (_i32, [_p, _i64, _p, _p, _i64, _i64, _p, _p]),
    "smlm_host_rows_add": (_i32, [_p, _p, _p, _i64, _p, _p, _p, _i64, _i64, _p, _p]),
    "smlm_rows_rowwise_step": (_i32, [_p, _i64, _p, _p, _p, _i64, _i64, _p, _p, _i32, _f32, _f32, _f32, _p, _f32,
                                      _i32, _p, _p]),
}

_LIB = None


def load(path=LIB_PATH):
    """The loaded library (once per process). Raises if the .so is missing or lacks an entry point."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                          "or `make -C sparse-memory-lm_b200/csrc`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)          # AttributeError names a missing export
        fn.restype, fn.argtypes = res, args
    _LIB = lib
    return lib


def lib():
    return _LIB if _LIB is not None else load()


def check(rc, what):
    if rc == OK:
        return
    msg = f"{what}: {lib().smlm_last_error().decode(errors='replace')}"
    if rc == ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


def dtype_code(dtype):
    if dtype == torch.float32:
        return F32
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float16:
        return F16
    raise ValueError(f"unsupported dtype {dtype} (fp32 / bf16 only)")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    """All given tensors (None skipped) on one CUDA device; returns it. No CPU path exists."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("smlm_b200 kernels run on CUDA tensors only (there is no CPU fallback); got a tensor "
                             f"on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


_STATUS = {}

# Optional per-call timing for benchmarks: set PROFILE to a list and every kernel entry appends
# (name, start_event, end_event, kernel_launches) recorded on the current stream around the call.
PROFILE = None
NVTX = os.environ.get("SMLM_B200_NVTX", "0") == "1"


class timed:
    """Context manager around one entry-point call: CUDA events when PROFILE is a list, an NVTX range when NVTX is
    on."""

    def __init__(self, name, launches):
        self.name, self.launches = name, launches

    def __enter__(self):
        self.nvtx = NVTX
        if self.nvtx:
            torch.cuda.nvtx.range_push(f"smlm:{self.name}")
        if PROFILE is not None:
            self.s = torch.cuda.Event(enable_timing=True)
            self.s.record()
        return self

    def __exit__(self, *exc):
        if PROFILE is not None and exc[0] is None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            PROFILE.append((self.name, self.s, e, self.launches))
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
        return False


def checked():
    return os.environ.get("SMLM_B200_CHECK", "0") == "1"


def status_ptr(device):
    """Device status word for out-of-range indices (allocated outside graph capture, else no status)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _STATUS.get(idx)
    if st is None:
        if torch.cuda.is_current_stream_capturing():
            return None
        st = _STATUS[idx] = torch.zeros(1, dtype=torch.int32, device=device)
    return ctypes.c_void_p(st.data_ptr())


def read_status(device, reset=True):
    """Flags raised on `device` since the last reset (synchronises the device)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _STATUS.get(idx)
    if st is None:
        return 0
    v = int(st.item())
    if reset:
        st.zero_()
    return v


def after(device, what):
    """Checked mode: synchronise and turn device status flags into exceptions."""
    if not checked() or torch.cuda.is_current_stream_capturing():
        return
    torch.cuda.synchronize(device)
    flags = read_status(device)
    if flags & FLAG_TIMEOUT:
        raise RuntimeError(f"{what}: a kernel-internal wait timed out (device status {flags:#x}); outputs invalid")
    if flags & FLAG_INDEX_RANGE:
        raise IndexError(f"{what}: row index out of range (device status {flags:#x})")
