// Helpers of the row-sharded value table: ordered sum of the owners' partial results, and the exchange of
// lookups, partial bags and weight gradients through peer memory.
#include <cstring>

#include "common.cuh"

namespace smlm {

// dst[i] = sum over s in order of src[s][i]; float4 lanes when count and both pointers allow.
template <int VEC>
__global__ void __launch_bounds__(256) slot_sum_kernel(const float* src, int64_t slots, int64_t count, float* dst) {
    const int64_t groups = count / VEC;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups;
         g += (int64_t)gridDim.x * blockDim.x) {
        if constexpr (VEC == 4) {
            float4 t = __ldg(reinterpret_cast<const float4*>(src) + g);
            for (int64_t s = 1; s < slots; s++) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(src + s * count) + g);
                t.x = t.x + x.x; t.y = t.y + x.y; t.z = t.z + x.z; t.w = t.w + x.w;
            }
            reinterpret_cast<float4*>(dst)[g] = t;
        } else {
            float t = __ldg(src + g);
            for (int64_t s = 1; s < slots; s++) t = t + __ldg(src + s * count + g);
            dst[g] = t;
        }
    }
}

// ------------------------------------------------------------------- exchange over peer memory (NVLink)
// Every rank owns one exchange block in its own HBM, mapped into the other ranks' address spaces (CUDA IPC; no
// multicast objects). Layout (offsets in XchgLayout): flags (int64, [4 kinds][world]: peers write their epoch
// into slot [kind][their rank]), a completion counter for this rank's kernels, the rank's lookups (int32 rows,
// fp32 weights, n_cap x k each; peers read them), the partial-bag receive area ([world][n_cap][d] fp32; owner o
// writes slot o) and the weight-gradient receive area (n_cap x k fp32; each lookup written by its owner).
// Protocol per step (epoch e, one outstanding forward per exchange):
//   forward  rank r copies its lookups into its block, zeroes its weight-gradient area, publishes
//            LOOKUPS[r] = e at every peer; each owner's fused kernel waits for LOOKUPS[s] >= e, reads rank s's
//            lookups over NVLink, gathers the rows it owns and stores the partial bag straight into rank s's
//            receive slot (peer stores), keeping a local copy of the lookups for the backward; its last CTA
//            publishes PARTIALS[o] = e at every rank after a system-scope fence; rank s waits for PARTIALS[o] >= e
//            from every owner and sums the slots in owner order.
//   backward each owner computes the weight gradients of its lookups from the all-gathered output gradients
//            and stores them straight into the requesting rank's area; GW[o] = e as above; the requester waits.
// Every wait is bounded (ten seconds of %globaltimer): on timeout the kernel raises SMLM_FLAG_TIMEOUT in the
// status word and stops waiting (outputs invalid); nothing traps.
constexpr int XK_LOOKUPS = 0, XK_PARTIALS = 1, XK_GW = 2;
constexpr uint64_t XCHG_WAIT_NS = 10000000000ull;  // 10 s: ranks may drift apart in warm-up

struct XchgLayout {
    size_t flags, counter, idx, w, partial, gw, total;
};

static XchgLayout xchg_layout(int world, int64_t n_cap, int64_t k, int64_t d) {
    XchgLayout L;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        off = (off + 255) & ~size_t(255);
        const size_t at = off;
        off += bytes;
        return at;
    };
    L.flags = take(sizeof(int64_t) * 4 * world);
    L.counter = take(sizeof(int) * 4);
    L.idx = take(sizeof(int32_t) * n_cap * k);
    L.w = take(sizeof(float) * n_cap * k);
    L.partial = take(sizeof(float) * world * n_cap * d);
    L.gw = take(sizeof(float) * n_cap * k);
    L.total = (off + 255) & ~size_t(255);
    return L;
}

__device__ __forceinline__ uint64_t xchg_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
    int64_t v;
    asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
    asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait of one thread for *f >= v; false (and SMLM_FLAG_TIMEOUT) when it gives up. A timeout seen in the
// status word (raised by any waiter of this or an earlier call) ends every later wait at once, so a broken
// exchange fails in one wait period instead of one per wave of blocks.
__device__ bool xchg_wait(const int64_t* f, int64_t v, int* status) {
    if (ld_acquire_sys(f) >= v) return true;
    const uint64_t t0 = xchg_now();
    while (ld_acquire_sys(f) < v) {
        if ((*reinterpret_cast<volatile int*>(status) & SMLM_FLAG_TIMEOUT) || xchg_now() - t0 > XCHG_WAIT_NS) {
            flag(status, SMLM_FLAG_TIMEOUT);
            return false;
        }
        __nanosleep(256);
    }
    return true;
}

struct XchgArgs {
    unsigned char* const* peers;  // (world,) device array: every rank's exchange block, this rank's included
    XchgLayout L;
    int rank, world;
    int64_t n, n_cap;
    int k, d;
    int64_t epoch;
    int* status;
};

__device__ __forceinline__ int64_t* xflag(const XchgArgs& x, int peer, int kind, int slot) {
    return reinterpret_cast<int64_t*>(x.peers[peer] + x.L.flags) + kind * x.world + slot;
}

// One block: FLAGS[kind][rank] = epoch at every rank, after a system-scope fence (the data it announces was
// written by earlier work on this stream).
__global__ void xchg_publish_kernel(XchgArgs x, int kind) {
    __threadfence_system();
    for (int p = threadIdx.x; p < x.world; p += blockDim.x) st_release_sys(xflag(x, p, kind, x.rank), x.epoch);
}

// Grid-wide completion: every CTA fences and counts in; the last one publishes FLAGS[kind][rank] = epoch at
// every rank and re-arms the counter.
__device__ void xchg_finish(const XchgArgs& x, int kind) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        int* counter = reinterpret_cast<int*>(x.peers[x.rank] + x.L.counter) + kind;
        if (atomicAdd(counter, 1) == (int)gridDim.x - 1) {
            __threadfence_system();
            for (int p = 0; p < x.world; p++) st_release_sys(xflag(x, p, kind, x.rank), x.epoch);
            atomicExch(counter, 0);
        }
    }
}

// Owner side of the forward: tasks (source rank s, token t, column block); the lookups of rank s are read from
// its exchange block (after LOOKUPS[s] >= epoch), the rows of this shard gathered as bag_gather_kernel does
// (same fmaf order over the token's in-shard lookups), the partial bag stored into rank s's receive slot
// [this rank][t]; the column-block-0 warp also keeps the lookups in all_idx / all_w (rows s n + t).
template <typename TT, int NS>
__global__ void __launch_bounds__(256) xchg_forward_kernel(XchgArgs x, const TT* table, int64_t row_base,
                                                           int64_t rows, int32_t* all_idx, float* all_w) {
    const int lane = lane_id();
    constexpr int CB = 32 * 4 * NS;
    const int nblk = (x.d + CB - 1) / CB;
    const int64_t tasks = (int64_t)x.world * x.n * nblk;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    int ready = -1;  // the source rank whose LOOKUPS flag this warp has seen
    bool ok = true;
    for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tasks && ok;
         task += warps) {
        const int s = (int)(task / (x.n * nblk));
        const int64_t rem = task % (x.n * nblk);
        const int64_t t = rem / nblk;
        const int c0 = (int)(rem % nblk) * CB;
        if (s != ready) {
            bool got = true;
            if (lane == 0) got = xchg_wait(xflag(x, x.rank, XK_LOOKUPS, s), x.epoch, x.status);
            ok = __shfl_sync(FULL, got, 0);
            __syncwarp();  // orders the other lanes' reads after lane 0's acquire
            if (!ok) break;
            ready = s;
        }
        const int32_t* sidx = reinterpret_cast<const int32_t*>(x.peers[s] + x.L.idx);
        const float* sw = reinterpret_cast<const float*>(x.peers[s] + x.L.w);
        float acc[NS][4];
#pragma unroll
        for (int q = 0; q < NS; q++) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
        for (int j0 = 0; j0 < x.k; j0 += 32) {
            const int cnt = min(32, x.k - j0);
            int64_t my_r = -1;
            float my_w = 0.f;
            if (lane < cnt) {
                const int64_t o = t * x.k + j0 + lane;
                const int32_t gi = __ldcg(sidx + o);  // another GPU's memory, rewritten every step: not via L1
                my_w = __ldcg(sw + o);
                if (c0 == 0) {
                    all_idx[(int64_t)s * x.n * x.k + o] = gi;
                    all_w[(int64_t)s * x.n * x.k + o] = my_w;
                }
                const int64_t r = (int64_t)gi - row_base;
                my_r = (r >= 0 && r < rows) ? r : -1;
            }
            unsigned todo = __ballot_sync(FULL, my_r >= 0);
            while (todo) {
                int64_t r[4];
                float wv[4];
                bool on[4];
                float v[4][NS][4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    on[u] = todo != 0;
                    const int src = on[u] ? __ffs(todo) - 1 : 0;
                    todo &= todo - 1;
                    r[u] = __shfl_sync(FULL, my_r, src);
                    wv[u] = __shfl_sync(FULL, my_w, src);
#pragma unroll
                    for (int q = 0; q < NS; q++) {
                        const int col = c0 + (lane + 32 * q) * 4;
                        if (on[u] && col < x.d) Elt<TT>::template load<4>(table + r[u] * x.d + col, v[u][q]);
                        else v[u][q][0] = v[u][q][1] = v[u][q][2] = v[u][q][3] = 0.f;
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; u++)
#pragma unroll
                    for (int q = 0; q < NS; q++)
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            if (on[u]) acc[q][i] = fmaf(wv[u], v[u][q][i], acc[q][i]);
            }
        }
        float* dst = reinterpret_cast<float*>(x.peers[s] + x.L.partial) + ((int64_t)x.rank * x.n_cap + t) * x.d;
#pragma unroll
        for (int q = 0; q < NS; q++) {
            const int col = c0 + (lane + 32 * q) * 4;
            if (col < x.d)
                *reinterpret_cast<float4*>(dst + col) = make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
        }
    }
    xchg_finish(x, XK_PARTIALS);
}

// Requester side: waits for PARTIALS[o] >= epoch from every owner, then out = slot sum in owner order.
__global__ void __launch_bounds__(256) xchg_sum_kernel(XchgArgs x, float* out) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        bool all = true;
        for (int o = 0; o < x.world && all; o++) all = xchg_wait(xflag(x, x.rank, XK_PARTIALS, o), x.epoch, x.status);
        ok = all;
    }
    __syncthreads();
    if (!ok) return;
    const float* src = reinterpret_cast<const float*>(x.peers[x.rank] + x.L.partial);
    const int64_t count = x.n * x.d;
    const int64_t slot = x.n_cap * x.d;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count / 4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 t = __ldcg(reinterpret_cast<const float4*>(src) + i);  // written by the peers: not via L1
        for (int o = 1; o < x.world; o++) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src + o * slot) + i);
            t.x = t.x + v.x; t.y = t.y + v.y; t.z = t.z + v.z; t.w = t.w + v.w;
        }
        reinterpret_cast<float4*>(out)[i] = t;
    }
}

// Owner side of the backward's weight gradient: bb_gw_kernel over every rank's tokens (output gradients
// all-gathered into g_all, lookups from the forward's local copy), each dot of an in-shard lookup stored
// straight into the requesting rank's weight-gradient area.
template <typename TT, typename GT, int NS>
__global__ void __launch_bounds__(128) xchg_gw_kernel(XchgArgs x, const GT* g_all, const int32_t* all_idx,
                                                      const TT* table, int64_t row_base, int64_t rows) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < x.world * x.n;
         task += warps) {
        const int s = (int)(task / x.n);
        const int64_t t = task % x.n;
        float gv[NS][4];
#pragma unroll
        for (int q = 0; q < NS; q++) {
            const int col = (lane + 32 * q) * 4;
            if (col < x.d) Elt<GT>::template load<4>(g_all + task * x.d + col, gv[q]);
            else gv[q][0] = gv[q][1] = gv[q][2] = gv[q][3] = 0.f;
        }
        float* dst = reinterpret_cast<float*>(x.peers[s] + x.L.gw) + t * x.k;
        for (int j0 = 0; j0 < x.k; j0 += 32) {
            const int cnt = min(32, x.k - j0);
            int64_t my_r = -1;
            if (lane < cnt) {
                const int64_t r = (int64_t)all_idx[task * x.k + j0 + lane] - row_base;
                my_r = (r >= 0 && r < rows) ? r : -1;
            }
            unsigned todo = __ballot_sync(FULL, my_r >= 0);
            const unsigned owned = todo;
            float mine = 0.f;
            while (todo) {
                int src[4];
                float v[4][NS][4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    src[u] = todo ? __ffs(todo) - 1 : -1;
                    if (todo) todo &= todo - 1;
                    const int64_t r = __shfl_sync(FULL, my_r, src[u] < 0 ? 0 : src[u]);
#pragma unroll
                    for (int q = 0; q < NS; q++) {
                        const int col = (lane + 32 * q) * 4;
                        if (src[u] >= 0 && col < x.d) Elt<TT>::template load<4>(table + r * x.d + col, v[u][q]);
                        else v[u][q][0] = v[u][q][1] = v[u][q][2] = v[u][q][3] = 0.f;
                    }
                }
                float dot[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    dot[u] = 0.f;
#pragma unroll
                    for (int q = 0; q < NS; q++)
#pragma unroll
                        for (int i = 0; i < 4; i++) dot[u] = fmaf(gv[q][i], v[u][q][i], dot[u]);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int u = 0; u < 4; u++) dot[u] += __shfl_xor_sync(FULL, dot[u], o);
#pragma unroll
                for (int u = 0; u < 4; u++)
                    if (lane == src[u]) mine = dot[u];
            }
            if (lane < cnt && (owned >> lane & 1u)) dst[j0 + lane] = mine;
        }
    }
    xchg_finish(x, XK_GW);
}

// Requester side of the weight gradient: waits for GW[o] >= epoch from every owner, copies the area to gw.
__global__ void __launch_bounds__(256) xchg_gw_collect_kernel(XchgArgs x, float* gw) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        bool all = true;
        for (int o = 0; o < x.world && all; o++) all = xchg_wait(xflag(x, x.rank, XK_GW, o), x.epoch, x.status);
        ok = all;
    }
    __syncthreads();
    if (!ok) return;
    const float* src = reinterpret_cast<const float*>(x.peers[x.rank] + x.L.gw);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < x.n * x.k; i += (int64_t)gridDim.x * blockDim.x)
        gw[i] = __ldcg(src + i);
}

}  // namespace smlm

using namespace smlm;

extern "C" size_t smlm_xchg_bytes(int world, int64_t n_cap, int64_t k, int64_t d) {
    if (world < 1 || n_cap < 0 || k < 0 || d < 0) return 0;
    return xchg_layout(world, n_cap, k, d).total;
}

extern "C" int smlm_xchg_alloc(size_t bytes, void** base, void* ipc_handle) {
    SMLM_CHECK_ARG(bytes > 0 && base && ipc_handle, "xchg_alloc: bad arguments");
    *base = nullptr;
    SMLM_CUDA(cudaMalloc(base, bytes));
    SMLM_CUDA(cudaMemset(*base, 0, bytes));
    cudaIpcMemHandle_t h;
    SMLM_CUDA(cudaIpcGetMemHandle(&h, *base));
    memcpy(ipc_handle, &h, sizeof(h));
    return SMLM_OK;
}

extern "C" int smlm_xchg_open(const void* ipc_handle, void** base) {
    SMLM_CHECK_ARG(ipc_handle && base, "xchg_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    SMLM_CUDA(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
    return SMLM_OK;
}

extern "C" int smlm_xchg_close(void* base) {
    if (base) SMLM_CUDA(cudaIpcCloseMemHandle(base));
    return SMLM_OK;
}

extern "C" int smlm_xchg_free(void* base) {
    if (base) SMLM_CUDA(cudaFree(base));
    return SMLM_OK;
}

static int xchg_args(XchgArgs* x, void* const* peers_dev, int rank, int world, int64_t n, int64_t n_cap, int64_t k,
                     int64_t d, int64_t epoch, int* status) {
    SMLM_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "xchg: bad rank %d of %d", rank, world);
    SMLM_CHECK_ARG(n >= 0 && n <= n_cap && k > 0 && k < (1 << 20) && d > 0 && d % 4 == 0 && d <= 512,
                   "xchg: bad sizes (n %lld, n_cap %lld, k %lld, d %lld; d must be a multiple of 4, at most 512)",
                   (long long)n, (long long)n_cap, (long long)k, (long long)d);
    SMLM_CHECK_ARG(peers_dev != nullptr && epoch > 0, "xchg: no peer table or epoch <= 0");
    SMLM_CHECK_ARG(status != nullptr, "xchg: the status word is required (it carries timeouts between waiters)");
    *x = XchgArgs{reinterpret_cast<unsigned char* const*>(peers_dev), xchg_layout(world, n_cap, k, d), rank, world, n,
                  n_cap, (int)k, (int)d, epoch, status};
    return SMLM_OK;
}

extern "C" int smlm_xchg_forward(void* const* peers_dev, void* my_block, int rank, int world, const int32_t* idx,
                                 const float* weights, int64_t n, int64_t k, int64_t n_cap, const void* table_shard,
                                 int table_dtype, int64_t row_base, int64_t shard_rows, int64_t d, int32_t* all_idx,
                                 float* all_w, float* out, int64_t epoch, int* status, void* stream) {
    XchgArgs x;
    int rc = xchg_args(&x, peers_dev, rank, world, n, n_cap, k, d, epoch, status);
    if (rc != SMLM_OK) return rc;
    SMLM_CHECK_ARG(table_dtype == SMLM_F32 || table_dtype == SMLM_BF16, "xchg_forward: table must be fp32 or bf16");
    SMLM_CHECK_ARG(my_block && all_idx && all_w && out && (n == 0 || (idx && weights)) &&
                   (table_shard || shard_rows == 0), "xchg_forward: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(table_shard) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0,
                   "xchg_forward: table and out must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    unsigned char* mine = static_cast<unsigned char*>(my_block);
    if (n > 0) {
        SMLM_CUDA(cudaMemcpyAsync(mine + x.L.idx, idx, sizeof(int32_t) * n * k, cudaMemcpyDeviceToDevice, st));
        SMLM_CUDA(cudaMemcpyAsync(mine + x.L.w, weights, sizeof(float) * n * k, cudaMemcpyDeviceToDevice, st));
    }
    SMLM_CUDA(cudaMemsetAsync(mine + x.L.gw, 0, sizeof(float) * n_cap * k, st));
    xchg_publish_kernel<<<1, 32, 0, st>>>(x, XK_LOOKUPS);
    SMLM_LAUNCHED("xchg_publish_kernel");
    const int ns = (int)((d + 127) / 128);
    const int64_t tasks = (int64_t)world * n;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((tasks + 7) / 8, (int64_t)sm_count() * 16));
    auto go = [&](auto NSc) {
        constexpr int NS = decltype(NSc)::value;
        if (table_dtype == SMLM_F32)
            xchg_forward_kernel<float, NS><<<blocks, 256, 0, st>>>(x, static_cast<const float*>(table_shard), row_base,
                                                                   shard_rows, all_idx, all_w);
        else
            xchg_forward_kernel<__nv_bfloat16, NS><<<blocks, 256, 0, st>>>(
                x, static_cast<const __nv_bfloat16*>(table_shard), row_base, shard_rows, all_idx, all_w);
    };
    if (ns <= 1) go(std::integral_constant<int, 1>{});
    else if (ns == 2) go(std::integral_constant<int, 2>{});
    else if (ns == 3) go(std::integral_constant<int, 3>{});
    else go(std::integral_constant<int, 4>{});
    SMLM_LAUNCHED("xchg_forward_kernel");
    const int sblocks = (int)std::max<int64_t>(1, std::min<int64_t>((n * d / 4 + 255) / 256, (int64_t)sm_count() * 8));
    xchg_sum_kernel<<<sblocks, 256, 0, st>>>(x, out);
    SMLM_LAUNCHED("xchg_sum_kernel");
    return SMLM_OK;
}

extern "C" int smlm_xchg_backward_gw(void* const* peers_dev, int rank, int world, const void* grad_all, int grad_dtype,
                                     const int32_t* all_idx, int64_t n, int64_t k, int64_t n_cap,
                                     const void* table_shard, int table_dtype, int64_t row_base, int64_t shard_rows,
                                     int64_t d, int64_t epoch, int* status, void* stream) {
    XchgArgs x;
    int rc = xchg_args(&x, peers_dev, rank, world, n, n_cap, k, d, epoch, status);
    if (rc != SMLM_OK) return rc;
    SMLM_CHECK_ARG(table_dtype == SMLM_F32 || table_dtype == SMLM_BF16, "xchg_backward_gw: table must be fp32 or bf16");
    SMLM_CHECK_ARG(grad_dtype == SMLM_F32 || grad_dtype == SMLM_BF16, "xchg_backward_gw: grad must be fp32 or bf16");
    SMLM_CHECK_ARG((n == 0 || (grad_all && all_idx)) && (table_shard || shard_rows == 0),
                   "xchg_backward_gw: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(table_shard) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(grad_all) % 16 == 0, "xchg_backward_gw: 16-byte alignment needed");
    cudaStream_t st = as_stream(stream);
    const int ns = (int)((d + 127) / 128);
    const int64_t tasks = (int64_t)world * n;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((tasks + 3) / 4, (int64_t)sm_count() * 32));
    auto go = [&](auto NSc) {
        constexpr int NS = decltype(NSc)::value;
        if (table_dtype == SMLM_F32) {
            const float* t = static_cast<const float*>(table_shard);
            if (grad_dtype == SMLM_F32)
                xchg_gw_kernel<float, float, NS><<<blocks, 128, 0, st>>>(x, static_cast<const float*>(grad_all), all_idx,
                                                                         t, row_base, shard_rows);
            else
                xchg_gw_kernel<float, __nv_bfloat16, NS><<<blocks, 128, 0, st>>>(
                    x, static_cast<const __nv_bfloat16*>(grad_all), all_idx, t, row_base, shard_rows);
        } else {
            const __nv_bfloat16* t = static_cast<const __nv_bfloat16*>(table_shard);
            if (grad_dtype == SMLM_F32)
                xchg_gw_kernel<__nv_bfloat16, float, NS><<<blocks, 128, 0, st>>>(
                    x, static_cast<const float*>(grad_all), all_idx, t, row_base, shard_rows);
            else
                xchg_gw_kernel<__nv_bfloat16, __nv_bfloat16, NS><<<blocks, 128, 0, st>>>(
                    x, static_cast<const __nv_bfloat16*>(grad_all), all_idx, t, row_base, shard_rows);
        }
    };
    if (ns <= 1) go(std::integral_constant<int, 1>{});
    else if (ns == 2) go(std::integral_constant<int, 2>{});
    else if (ns == 3) go(std::integral_constant<int, 3>{});
    else go(std::integral_constant<int, 4>{});
    SMLM_LAUNCHED("xchg_gw_kernel");
    return SMLM_OK;
}

extern "C" int smlm_xchg_collect_gw(void* const* peers_dev, int rank, int world, int64_t n, int64_t k, int64_t n_cap,
                                    int64_t d, float* gw, int64_t epoch, int* status, void* stream) {
    XchgArgs x;
    int rc = xchg_args(&x, peers_dev, rank, world, n, n_cap, k, d, epoch, status);
    if (rc != SMLM_OK) return rc;
    SMLM_CHECK_ARG(gw || n == 0, "xchg_collect_gw: null pointer");
    const int cblocks = (int)std::max<int64_t>(1, std::min<int64_t>((n * k + 255) / 256, (int64_t)sm_count() * 8));
    xchg_gw_collect_kernel<<<cblocks, 256, 0, as_stream(stream)>>>(x, gw);
    SMLM_LAUNCHED("xchg_gw_collect_kernel");
    return SMLM_OK;
}

extern "C" int smlm_slot_sum(const float* src, int64_t slots, int64_t count, float* dst, void* stream) {
    SMLM_CHECK_ARG(slots >= 1 && count >= 0, "slot_sum: bad sizes");
    if (count == 0) return SMLM_OK;
    SMLM_CHECK_ARG(src && dst, "slot_sum: null pointer");
    const bool vec = count % 4 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(dst) % 16 == 0;
    const int64_t groups = vec ? count / 4 : count;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((groups + 255) / 256, (int64_t)sm_count() * 8));
    if (vec) slot_sum_kernel<4><<<blocks, 256, 0, as_stream(stream)>>>(src, slots, count, dst);
    else slot_sum_kernel<1><<<blocks, 256, 0, as_stream(stream)>>>(src, slots, count, dst);
    SMLM_LAUNCHED("slot_sum_kernel");
    return SMLM_OK;
}
