// Helpers of the row-sharded value table: ordered sum of the owners' partial results, and the exchange of
// lookups, partial bags and weight gradients through peer memory.
#include <cstring>

#include <cub/device/device_scan.cuh>

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
// multicast objects). Layout (XchgLayout): flags (int64, [3 kinds][world]: peers write their epoch into slot
// [kind][their rank]), completion counters, this rank's current epoch, its lookups bucketed by owner (the CSR
// below; peers read their bucket), the partial-bag receive area ([world][n_cap][d] fp32; owner o writes slot o)
// and the weight-gradient receive area (n_cap x k fp32; each lookup written by its owner).
//
// Owner buckets (CSR over (owner, token)): cnt[o * n + t] = how many of token t's lookups rank o's rows hold;
// off = its exclusive prefix sum (off[world * n] = all valid lookups), so owner o's lookups of token t are
// entries [off[o n + t], off[o n + t + 1]) of lk_row (row local to the owner's shard), lk_w (weight) and lk_pos
// (t k + the lookup's slot in the token), in slot order; a range of tokens is one contiguous range of entries.
// Owner o reads only its own bucket of every rank: about n k / world lookups per rank instead of all n k.
//
// Protocol per step (epoch e, one outstanding forward per exchange):
//   forward  rank r buckets its lookups by owner into its block, zeroes its weight-gradient area and publishes
//            LOOKUPS[r] = e at every peer; each owner's fused kernel waits for LOOKUPS[s] >= e, reads its bucket
//            of rank s over NVLink, gathers its rows and stores the partial bag straight into rank s's receive
//            slot (peer stores), keeping a dense local copy of the lookups it served for the backward (rows of
//            other owners -1); its last CTA publishes PARTIALS[o] = e at every rank after a system-scope fence;
//            rank s waits for PARTIALS[o] >= e from every owner and sums the slots in owner order (optionally
//            times silu(pre), the swilu product, and rounded to bf16).
//   backward each owner computes the weight gradients of its lookups from the all-gathered output gradients
//            and stores them straight into the requesting rank's area; GW[o] = e as above; the requester waits.
// Epochs: a caller may pass one (> 0); with 0 the forward advances the block's own counter on the device, and the
// backward uses the forward's, so a step replayed from a CUDA graph gets a new epoch on every replay (every rank
// runs the same exchanges in the same order, so the counters agree).
// Every wait is bounded (ten seconds of %globaltimer): on timeout the kernel raises SMLM_FLAG_TIMEOUT in the
// status word and stops waiting (outputs invalid); nothing traps.
constexpr int XK_LOOKUPS = 0, XK_PARTIALS = 1, XK_GW = 2, XK_KINDS = 3;
constexpr uint64_t XCHG_WAIT_NS = 10000000000ull;  // 10 s: ranks may drift apart in warm-up
constexpr int XCHG_MAX_WORLD = 64;

struct XchgLayout {
    size_t flags, counter, epoch, cnt, off, lk_row, lk_w, lk_pos, scan_tmp, scan_tmp_bytes, partial, gw, total;
};

static size_t xchg_scan_bytes(int64_t items) {
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, (const int32_t*)nullptr, (int32_t*)nullptr,
                                  (int)std::max<int64_t>(items, 1));
    return bytes;
}

static XchgLayout xchg_layout(int world, int64_t n_cap, int64_t k, int64_t d) {
    XchgLayout L;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        off = (off + 255) & ~size_t(255);
        const size_t at = off;
        off += bytes;
        return at;
    };
    const int64_t buckets = (int64_t)world * n_cap + 1;
    L.flags = take(sizeof(int64_t) * XK_KINDS * world);
    L.counter = take(sizeof(int) * 4);
    L.epoch = take(sizeof(int64_t));
    L.cnt = take(sizeof(int32_t) * buckets);
    L.off = take(sizeof(int32_t) * buckets);
    L.lk_row = take(sizeof(int32_t) * n_cap * k);
    L.lk_w = take(sizeof(float) * n_cap * k);
    L.lk_pos = take(sizeof(int32_t) * n_cap * k);
    L.scan_tmp_bytes = xchg_scan_bytes(buckets);
    L.scan_tmp = take(L.scan_tmp_bytes);
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
    int64_t epoch_host;  // > 0: the caller's epoch; 0: the block's device counter
    int* status;
};

__device__ __forceinline__ int64_t* xflag(const XchgArgs& x, int peer, int kind, int slot) {
    return reinterpret_cast<int64_t*>(x.peers[peer] + x.L.flags) + kind * x.world + slot;
}

// The exchange's current epoch (the caller's, or the one the last forward set in this rank's block).
__device__ __forceinline__ int64_t xchg_epoch(const XchgArgs& x) {
    if (x.epoch_host > 0) return x.epoch_host;
    return *reinterpret_cast<const volatile int64_t*>(x.peers[x.rank] + x.L.epoch);
}

template <typename T>
__device__ __forceinline__ T* xarea(const XchgArgs& x, int peer, size_t at) {
    return reinterpret_cast<T*>(x.peers[peer] + at);
}

// Owner of a global row (-1: a padding lookup, row < 0; past the last shard: flagged, skipped).
__device__ __forceinline__ int xchg_owner(int32_t row, int64_t per, int world, int* status) {
    if (row < 0) return -1;
    const int64_t o = (int64_t)row / per;
    if (o >= world) {
        flag(status, SMLM_FLAG_INDEX_RANGE);
        return -1;
    }
    return (int)o;
}

// Requester, pass 1 (one warp per token): cnt[o * n + t] = the token's lookups held by owner o; cnt[world n] = 0
// (so that the exclusive scan's last entry is the total).
__global__ void __launch_bounds__(256) xchg_count_kernel(XchgArgs x, const int32_t* idx, int64_t per) {
    __shared__ int counts[8][XCHG_MAX_WORLD];
    const int lane = lane_id(), wib = threadIdx.x >> 5;
    int* c = counts[wib];
    int32_t* cnt = xarea<int32_t>(x, x.rank, x.L.cnt);
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    if (blockIdx.x == 0 && threadIdx.x == 0) cnt[(int64_t)x.world * x.n] = 0;
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + wib; t < x.n; t += warps) {
        for (int o = lane; o < x.world; o += 32) c[o] = 0;
        __syncwarp();
        for (int j0 = 0; j0 < x.k; j0 += 32) {
            int o = -1;
            if (j0 + lane < x.k) o = xchg_owner(idx[t * x.k + j0 + lane], per, x.world, x.status);
            const unsigned same = __match_any_sync(FULL, o);
            if (o >= 0 && lane == __ffs(same) - 1) c[o] += __popc(same);
            __syncwarp();
        }
        for (int o = lane; o < x.world; o += 32) cnt[(int64_t)o * x.n + t] = c[o];
        __syncwarp();
    }
}

// Requester, pass 2 (one warp per token): each lookup into its owner's bucket at off[o n + t] + (its rank among
// the token's lookups of that owner, in slot order).
__global__ void __launch_bounds__(256) xchg_scatter_kernel(XchgArgs x, const int32_t* idx, const float* w,
                                                           int64_t per) {
    __shared__ int next[8][XCHG_MAX_WORLD];
    const int lane = lane_id(), wib = threadIdx.x >> 5;
    int* pos = next[wib];
    const int32_t* off = xarea<const int32_t>(x, x.rank, x.L.off);
    int32_t* lk_row = xarea<int32_t>(x, x.rank, x.L.lk_row);
    float* lk_w = xarea<float>(x, x.rank, x.L.lk_w);
    int32_t* lk_pos = xarea<int32_t>(x, x.rank, x.L.lk_pos);
    const unsigned below = (1u << lane) - 1u;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + wib; t < x.n; t += warps) {
        for (int o = lane; o < x.world; o += 32) pos[o] = off[(int64_t)o * x.n + t];
        __syncwarp();
        for (int j0 = 0; j0 < x.k; j0 += 32) {
            const int j = j0 + lane;
            int o = -1;
            int32_t row = -1;
            if (j < x.k) {
                row = idx[t * x.k + j];
                o = row < 0 || (int64_t)row / per >= x.world ? -1 : (int)((int64_t)row / per);
            }
            const unsigned same = __match_any_sync(FULL, o);
            if (o >= 0) {
                const int64_t q = pos[o] + __popc(same & below);
                lk_row[q] = (int32_t)(row - (int64_t)o * per);
                lk_w[q] = w[t * x.k + j];
                lk_pos[q] = (int32_t)(t * x.k + j);
            }
            __syncwarp();
            if (o >= 0 && lane == __ffs(same) - 1) pos[o] += __popc(same);
            __syncwarp();
        }
    }
}

// One block: FLAGS[kind][rank] = epoch at every rank, after a system-scope fence (the data it announces was
// written by earlier work on this stream). advance: first set the block's epoch (the caller's, or one past the
// current) for the exchange that starts here.
__global__ void xchg_publish_kernel(XchgArgs x, int kind, int advance) {
    __shared__ int64_t e;
    if (threadIdx.x == 0) {
        int64_t* ep = xarea<int64_t>(x, x.rank, x.L.epoch);
        e = x.epoch_host > 0 ? x.epoch_host : *ep + (advance ? 1 : 0);
        if (advance) *ep = e;
    }
    __syncthreads();
    __threadfence_system();
    for (int p = threadIdx.x; p < x.world; p += blockDim.x) st_release_sys(xflag(x, p, kind, x.rank), e);
}

// Grid-wide completion: every CTA fences and counts in; the last one publishes FLAGS[kind][rank] = epoch at
// every rank and re-arms the counter.
__device__ void xchg_finish(const XchgArgs& x, int kind) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        int* counter = xarea<int>(x, x.rank, x.L.counter) + kind;
        if (atomicAdd(counter, 1) == (int)gridDim.x - 1) {
            __threadfence_system();
            const int64_t e = xchg_epoch(x);
            for (int p = 0; p < x.world; p++) st_release_sys(xflag(x, p, kind, x.rank), e);
            atomicExch(counter, 0);
        }
    }
}

// Owner side of the forward: tasks (source rank s, group of XG tokens, column block). This rank's bucket of rank
// s's lookups of the group's tokens is one contiguous range of entries of s's block (two offsets), read over
// NVLink 32 entries at a time (the next 32 in flight while the current ones are gathered); the rows are gathered
// four at a time and each token's lookups summed in slot order (fmaf, as bag_gather_kernel sums a token's
// lookups); every token's partial bag (zero when this shard holds none of its rows) is stored into rank s's
// receive slot [this rank][t]. With DENSE, the column-block-0 warp also writes the lookups it served into the dense
// local copy all_idx / all_w (row (s n + t) k + slot; the caller set the other slots to -1).
constexpr int XG = 4;  // tokens per task

template <typename TT, int NS, bool DENSE>
__global__ void __launch_bounds__(256, 2) xchg_forward_kernel(XchgArgs x, const TT* table, int64_t row_base,
                                                           int64_t rows, int32_t* all_idx, float* all_w) {
    const int lane = lane_id();
    constexpr int CB = 32 * 4 * NS;
    const int nblk = (x.d + CB - 1) / CB;
    const int64_t groups = (x.n + XG - 1) / XG;
    const int64_t tasks = (int64_t)x.world * groups * nblk;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t epoch = xchg_epoch(x);
    int ready = -1;  // the source rank whose LOOKUPS flag this warp has seen
    bool ok = true;
    for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tasks && ok;
         task += warps) {
        const int s = (int)(task / (groups * nblk));
        const int64_t rem = task % (groups * nblk);
        const int64_t t0 = (rem / nblk) * XG;
        const int64_t t1 = min(t0 + XG, x.n);
        const int c0 = (int)(rem % nblk) * CB;
        if (s != ready) {
            bool got = true;
            if (lane == 0) got = xchg_wait(xflag(x, x.rank, XK_LOOKUPS, s), epoch, x.status);
            ok = __shfl_sync(FULL, got, 0);
            __syncwarp();  // orders the other lanes' reads after lane 0's acquire
            if (!ok) break;
            ready = s;
        }
        // another GPU's memory, rewritten every step: read through L2 only
        const int32_t* soff = xarea<const int32_t>(x, s, x.L.off) + (int64_t)x.rank * x.n;
        int64_t bound = 0;
        if (lane < 2) bound = __ldcg(soff + (lane == 0 ? t0 : t1));
        const int64_t beg = __shfl_sync(FULL, bound, 0), end = __shfl_sync(FULL, bound, 1);
        const int32_t* srow = xarea<const int32_t>(x, s, x.L.lk_row);
        const float* sw = xarea<const float>(x, s, x.L.lk_w);
        const int32_t* spos = xarea<const int32_t>(x, s, x.L.lk_pos);
        float* dst = xarea<float>(x, s, x.L.partial) + (int64_t)x.rank * x.n_cap * x.d;
        float acc[NS][4];
#pragma unroll
        for (int q = 0; q < NS; q++) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
        int64_t cur = t0;  // the token whose partial acc holds
        auto store = [&]() {
#pragma unroll
            for (int q = 0; q < NS; q++) {
                const int col = c0 + (lane + 32 * q) * 4;
                if (col < x.d)
                    *reinterpret_cast<float4*>(dst + cur * x.d + col) =
                        make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
                acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
            }
            cur++;
        };
        // entries of the chunk at q0: lane l holds entry q0 + l (row local to this shard, weight, t k + slot)
        auto fetch = [&](int64_t q0, int32_t& r, float& wv, int32_t& pos) {
            r = -1;
            wv = 0.f;
            pos = 0;
            if (q0 + lane < end) {
                r = __ldcg(srow + q0 + lane);
                wv = __ldcg(sw + q0 + lane);
                pos = __ldcg(spos + q0 + lane);
            }
        };
        int32_t nr, np;
        float nw;
        fetch(beg, nr, nw, np);
        for (int64_t q0 = beg; q0 < end; q0 += 32) {
            const int cnt = (int)min((int64_t)32, end - q0);
            const int32_t my_r0 = nr, my_pos = np;
            const float my_w = nw;
            if (q0 + 32 < end) fetch(q0 + 32, nr, nw, np);  // the next chunk's entries in flight
            int64_t my_r = -1;
            if (lane < cnt) {
                if (my_r0 >= 0 && my_r0 < rows) my_r = my_r0;
                else flag(x.status, SMLM_FLAG_INDEX_RANGE);
                if (DENSE && c0 == 0) {
                    const int64_t o = (int64_t)s * x.n * x.k + my_pos;
                    all_idx[o] = my_r >= 0 ? (int32_t)(my_r + row_base) : -1;
                    all_w[o] = my_w;
                }
            }
            const int32_t my_r32 = (int32_t)my_r;
            for (int u0 = 0; u0 < cnt; u0 += 4) {
                int32_t r[4], tok[4];
                float wv[4];
                float v[4][NS][4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int src = min(u0 + u, cnt - 1);
                    r[u] = __shfl_sync(FULL, my_r32, src);
                    wv[u] = __shfl_sync(FULL, my_w, src);
                    tok[u] = __shfl_sync(FULL, my_pos, src) / x.k;
                    if (u0 + u >= cnt) r[u] = -2;  // past the chunk: nothing
#pragma unroll
                    for (int q = 0; q < NS; q++) {
                        const int col = c0 + (lane + 32 * q) * 4;
                        if (r[u] >= 0 && col < x.d)
                            Elt<TT>::template load<4>(table + (int64_t)r[u] * x.d + col, v[u][q]);
                        else v[u][q][0] = v[u][q][1] = v[u][q][2] = v[u][q][3] = 0.f;
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (r[u] == -2) continue;
                    while (cur < tok[u]) store();  // the tokens before this entry's are complete
                    if (r[u] >= 0) {
#pragma unroll
                        for (int q = 0; q < NS; q++)
#pragma unroll
                            for (int i = 0; i < 4; i++) acc[q][i] = fmaf(wv[u], v[u][q][i], acc[q][i]);
                    }
                }
            }
        }
        while (cur < t1) store();
    }
    xchg_finish(x, XK_PARTIALS);
}

// Requester side: waits for PARTIALS[o] >= epoch from every owner, then out = slot sum in owner order; with pre,
// times silu(pre) (the swilu product, as the inference bag applies it); stored as fp32 or bf16.
__global__ void __launch_bounds__(256) xchg_sum_kernel(XchgArgs x, const void* pre, int pre_dtype, void* out,
                                                       int out_dtype) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        const int64_t e = xchg_epoch(x);
        bool all = true;
        for (int o = 0; o < x.world && all; o++) all = xchg_wait(xflag(x, x.rank, XK_PARTIALS, o), e, x.status);
        ok = all;
    }
    __syncthreads();
    if (!ok) return;
    const float* src = xarea<const float>(x, x.rank, x.L.partial);
    const int64_t count = x.n * x.d;
    const int64_t slot = x.n_cap * x.d;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count / 4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 t = __ldcg(reinterpret_cast<const float4*>(src) + i);  // written by the peers: not via L1
        for (int o = 1; o < x.world; o++) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src + o * slot) + i);
            t.x = t.x + v.x; t.y = t.y + v.y; t.z = t.z + v.z; t.w = t.w + v.w;
        }
        float r[4] = {t.x, t.y, t.z, t.w};
        if (pre) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int64_t o = i * 4 + c;
                const float p = pre_dtype == SMLM_F32 ? __ldg(static_cast<const float*>(pre) + o)
                                                      : bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(pre) + o));
                r[c] = r[c] * silu_bf16(p);
            }
        }
        if (out_dtype == SMLM_F32) {
            reinterpret_cast<float4*>(out)[i] = make_float4(r[0], r[1], r[2], r[3]);
        } else {
            uint2 b;
            b.x = f32_to_bf16_bits(r[0]) | (f32_to_bf16_bits(r[1]) << 16);
            b.y = f32_to_bf16_bits(r[2]) | (f32_to_bf16_bits(r[3]) << 16);
            reinterpret_cast<uint2*>(out)[i] = b;
        }
    }
}

// Owner side of the backward's weight gradient: bb_gw_kernel over every rank's tokens (output gradients
// all-gathered into g_all, lookups from the forward's dense local copy), each dot of an in-shard lookup stored
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
        float* dst = xarea<float>(x, s, x.L.gw) + t * x.k;
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
        const int64_t e = xchg_epoch(x);
        bool all = true;
        for (int o = 0; o < x.world && all; o++) all = xchg_wait(xflag(x, x.rank, XK_GW, o), e, x.status);
        ok = all;
    }
    __syncthreads();
    if (!ok) return;
    const float* src = xarea<const float>(x, x.rank, x.L.gw);
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
    SMLM_CHECK_ARG(world >= 1 && world <= XCHG_MAX_WORLD && rank >= 0 && rank < world, "xchg: bad rank %d of %d "
                   "(at most %d ranks)", rank, world, XCHG_MAX_WORLD);
    SMLM_CHECK_ARG(n >= 0 && n <= n_cap && k > 0 && k < (1 << 20) && d > 0 && d % 4 == 0 && d <= 512 &&
                       (int64_t)world * n_cap < (1ll << 31) - 1 && n_cap * k < (1ll << 31),
                   "xchg: bad sizes (n %lld, n_cap %lld, k %lld, d %lld; d must be a multiple of 4, at most 512)",
                   (long long)n, (long long)n_cap, (long long)k, (long long)d);
    SMLM_CHECK_ARG(peers_dev != nullptr && epoch >= 0, "xchg: no peer table or epoch < 0");
    SMLM_CHECK_ARG(status != nullptr, "xchg: the status word is required (it carries timeouts between waiters)");
    *x = XchgArgs{reinterpret_cast<unsigned char* const*>(peers_dev), xchg_layout(world, n_cap, k, d), rank, world, n,
                  n_cap, (int)k, (int)d, epoch, status};
    return SMLM_OK;
}

extern "C" int smlm_xchg_forward(void* const* peers_dev, void* my_block, int rank, int world, const int32_t* idx,
                                 const float* weights, int64_t n, int64_t k, int64_t n_cap, int64_t rows_per_rank,
                                 const void* table_shard, int table_dtype, int64_t row_base, int64_t shard_rows,
                                 int64_t d, int32_t* all_idx, float* all_w, const void* pre, int pre_dtype, void* out,
                                 int out_dtype, int64_t epoch, int* status, void* stream) {
    XchgArgs x;
    int rc = xchg_args(&x, peers_dev, rank, world, n, n_cap, k, d, epoch, status);
    if (rc != SMLM_OK) return rc;
    SMLM_CHECK_ARG(table_dtype == SMLM_F32 || table_dtype == SMLM_BF16, "xchg_forward: table must be fp32 or bf16");
    SMLM_CHECK_ARG(out_dtype == SMLM_F32 || out_dtype == SMLM_BF16, "xchg_forward: out must be fp32 or bf16");
    SMLM_CHECK_ARG(pre == nullptr || pre_dtype == SMLM_F32 || pre_dtype == SMLM_BF16,
                   "xchg_forward: pre must be fp32 or bf16");
    SMLM_CHECK_ARG(rows_per_rank > 0 && shard_rows >= 0 && shard_rows <= rows_per_rank && row_base >= 0,
                   "xchg_forward: bad shard (rows_per_rank %lld, shard rows %lld)", (long long)rows_per_rank,
                   (long long)shard_rows);
    SMLM_CHECK_ARG((all_idx == nullptr) == (all_w == nullptr), "xchg_forward: all_idx and all_w go together");
    SMLM_CHECK_ARG(my_block && out && (n == 0 || (idx && weights)) && (table_shard || shard_rows == 0),
                   "xchg_forward: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(table_shard) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(pre) % 16 == 0,
                   "xchg_forward: table, pre and out must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    unsigned char* mine = static_cast<unsigned char*>(my_block);
    // this rank's lookups bucketed by owner (count, prefix sum, scatter) into its block
    const int wblocks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, (int64_t)sm_count() * 8));
    xchg_count_kernel<<<wblocks, 256, 0, st>>>(x, idx, rows_per_rank);
    SMLM_LAUNCHED("xchg_count_kernel");
    size_t scan_bytes = xchg_scan_bytes((int64_t)world * n + 1);
    SMLM_CHECK_ARG(scan_bytes <= x.L.scan_tmp_bytes, "xchg_forward: scan scratch too small");
    SMLM_CUDA(cub::DeviceScan::ExclusiveSum(mine + x.L.scan_tmp, scan_bytes,
                                            reinterpret_cast<const int32_t*>(mine + x.L.cnt),
                                            reinterpret_cast<int32_t*>(mine + x.L.off), (int)(world * n + 1), st));
    if (n > 0) {
        xchg_scatter_kernel<<<wblocks, 256, 0, st>>>(x, idx, weights, rows_per_rank);
        SMLM_LAUNCHED("xchg_scatter_kernel");
    }
    SMLM_CUDA(cudaMemsetAsync(mine + x.L.gw, 0, sizeof(float) * n_cap * k, st));
    if (all_idx && n > 0) SMLM_CUDA(cudaMemsetAsync(all_idx, 0xff, sizeof(int32_t) * world * n * k, st));
    xchg_publish_kernel<<<1, 32, 0, st>>>(x, XK_LOOKUPS, 1);
    SMLM_LAUNCHED("xchg_publish_kernel");
    const int ns = (int)((d + 127) / 128);
    const int64_t tasks = (int64_t)world * ((n + XG - 1) / XG);
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((tasks + 7) / 8, (int64_t)sm_count() * 16));
    auto go = [&](auto NSc, auto DENSEc) {
        constexpr int NS = decltype(NSc)::value;
        constexpr bool DENSE = decltype(DENSEc)::value;
        if (table_dtype == SMLM_F32)
            xchg_forward_kernel<float, NS, DENSE><<<blocks, 256, 0, st>>>(
                x, static_cast<const float*>(table_shard), row_base, shard_rows, all_idx, all_w);
        else
            xchg_forward_kernel<__nv_bfloat16, NS, DENSE><<<blocks, 256, 0, st>>>(
                x, static_cast<const __nv_bfloat16*>(table_shard), row_base, shard_rows, all_idx, all_w);
    };
    auto by_ns = [&](auto DENSEc) {
        if (ns <= 1) go(std::integral_constant<int, 1>{}, DENSEc);
        else if (ns == 2) go(std::integral_constant<int, 2>{}, DENSEc);
        else if (ns == 3) go(std::integral_constant<int, 3>{}, DENSEc);
        else go(std::integral_constant<int, 4>{}, DENSEc);
    };
    if (all_idx) by_ns(std::true_type{});
    else by_ns(std::false_type{});
    SMLM_LAUNCHED("xchg_forward_kernel");
    const int sblocks = (int)std::max<int64_t>(1, std::min<int64_t>((n * d / 4 + 255) / 256, (int64_t)sm_count() * 8));
    xchg_sum_kernel<<<sblocks, 256, 0, st>>>(x, pre, pre_dtype, out, out_dtype);
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
