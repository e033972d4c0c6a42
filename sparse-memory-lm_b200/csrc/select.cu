// Product-key selection on sub-key scores, its backward, and exact fp32 sub-key scoring.
//
// Selection order everywhere: score descending, then index ascending ("ties go to the lower index").
// Scores are compared through order-preserving integer codes packed with the inverted index into one u64 key
// (code << 32 | ~index), so one unsigned comparison implements the full order and every key of a row is
// distinct.
//
// Per (token, head) row, one warp:
//   1. each half: top-knn of nk scores. A threshold (the smallest of the 32 lanes' maxima, which at least
//      32 keys reach) filters the row into a shared-memory buffer; the survivors are bitonic-sorted.
//   2. the pairs (a, b) of the two sorted lists with (a+1)(b+1) <= knn: every other pair has at least knn
//      pairs that are >= it, so the knn-th best pair score T is exact; pairs with a score > T are all among
//      them. The pair sums are rounded to the score type (as `s1 + s2` in PyTorch) and sorted.
//   3. if a pair outside that set also scores exactly T (checked at the first excluded pair of every list
//      row, the only place one can appear), the entries with score T are re-chosen over the full knn x knn
//      product by lowest full index.
//   4. softmax in fp32 over the knn scores.
#include "common.cuh"

namespace smlm {

constexpr int SEL_CAP = 256;  // survivor buffer (u64 keys) per warp
constexpr int SEL_WARPS = 8;

template <bool F32>
__device__ __forceinline__ uint32_t score_bits(const void* s, int64_t i) {
    if constexpr (F32) return __float_as_uint(__ldg(static_cast<const float*>(s) + i));
    else return __ldg(static_cast<const uint16_t*>(s) + i);
}
template <bool F32>
__device__ __forceinline__ uint32_t code_of(uint32_t bits) {
    if constexpr (F32) return order_code32(bits);
    else return order_code16(bits);
}
template <bool F32>
__device__ __forceinline__ float score_of_code(uint32_t c) {
    if constexpr (F32) return __uint_as_float(decode_code32(c));
    else return bf16_bits_to_f32(decode_code16(c));
}
template <bool F32>
__device__ __forceinline__ uint32_t bits_of_float(float x) {
    if constexpr (F32) return __float_as_uint(x);
    else return f32_to_bf16_bits(x);
}
__device__ __forceinline__ uint64_t make_key(uint32_t code, uint32_t index) {
    return ((uint64_t)code << 32) | (uint64_t)(0xffffffffu - index);
}
__device__ __forceinline__ uint32_t key_index(uint64_t k) { return 0xffffffffu - (uint32_t)k; }
__device__ __forceinline__ uint32_t key_code(uint64_t k) { return (uint32_t)(k >> 32); }

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t x = __shfl_xor_sync(FULL, v, o);
        v = x < v ? x : v;
    }
    return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t x = __shfl_xor_sync(FULL, v, o);
        v = x > v ? x : v;
    }
    return v;
}

// Descending bitonic sort of buf[0, n), n a power of two, by one warp.
__device__ void warp_sort_desc(uint64_t* buf, int n) {
    const int lane = lane_id();
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < n; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t a = buf[i], b = buf[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        buf[i] = b;
                        buf[ixj] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
}

__device__ __forceinline__ int pow2_at_least(int n) {
    int p = 32;
    while (p < n) p <<= 1;
    return p;
}

// Sorts buf[0, cnt) descending (zero padding up to a power of two).
__device__ void sort_prefix(uint64_t* buf, int cnt) {
    const int lane = lane_id();
    const int n = pow2_at_least(cnt);
    for (int i = cnt + lane; i < n; i += 32) buf[i] = 0;
    __syncwarp();
    warp_sort_desc(buf, n);
}

// Top-knn keys of one half (nk scores at s + off) left sorted in buf[0, knn).
template <bool F32>
__device__ void half_topk(const void* s, int64_t off, int nk, int knn, uint64_t* buf) {
    const int lane = lane_id();
    uint64_t mx = 0;
    for (int k = lane; k < nk; k += 32) {
        const uint64_t key = make_key(code_of<F32>(score_bits<F32>(s, off + k)), (uint32_t)k);
        mx = key > mx ? key : mx;
    }
    uint64_t theta = warp_min_u64(mx);  // >= 32 keys (or all of them) are >= theta
    int cnt = 0;
    for (int base = 0; base < nk; base += 32) {
        const int k = base + lane;
        const uint64_t key = k < nk ? make_key(code_of<F32>(score_bits<F32>(s, off + k)), (uint32_t)k) : 0;
        unsigned pass = __ballot_sync(FULL, k < nk && key >= theta);
        if (cnt + __popc(pass) > SEL_CAP) {
            sort_prefix(buf, cnt);
            cnt = knn;
            theta = buf[knn - 1] + 1;  // keys are distinct: only strictly better ones from here on
            pass = __ballot_sync(FULL, k < nk && key >= theta);
        }
        if (pass & (1u << lane)) buf[cnt + __popc(pass & ((1u << lane) - 1))] = key;
        cnt += __popc(pass);
    }
    __syncwarp();
    sort_prefix(buf, cnt);
}

// Bitonic sort of one key per lane, descending across the warp.
__device__ __forceinline__ uint64_t warp_sort32_desc(uint64_t v, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint64_t o = __shfl_xor_sync(FULL, v, stride);
            const bool desc = (lane & size) == 0 || size == 32;
            const bool lower = (lane & stride) == 0;
            v = (lower == desc) ? (v > o ? v : o) : (v < o ? v : o);
        }
    }
    return v;
}

// Top 32 (descending, one per lane) of two descending lane sequences: max(a[i], b[31 - i]) is bitonic and holds
// the 32 largest; a half-cleaner network sorts it.
__device__ __forceinline__ uint64_t warp_merge_top32(uint64_t a, uint64_t b, int lane) {
    const uint64_t br = __shfl_sync(FULL, b, 31 - lane);
    uint64_t v = a > br ? a : br;
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) {
        const uint64_t o = __shfl_xor_sync(FULL, v, stride);
        v = (lane & stride) == 0 ? (v > o ? v : o) : (v < o ? v : o);
    }
    return v;
}

// The 32 largest of 128 keys (4 per lane), sorted descending, one per lane.
__device__ __forceinline__ uint64_t warp_top32_of_128(uint64_t (&k)[4], int lane) {
#pragma unroll
    for (int r = 0; r < 4; r++) k[r] = warp_sort32_desc(k[r], lane);
    return warp_merge_top32(warp_merge_top32(k[0], k[1], lane), warp_merge_top32(k[2], k[3], lane), lane);
}

template <bool F32>
__device__ __forceinline__ uint32_t pair_code(float v1, float v2) {
    return code_of<F32>(bits_of_float<F32>(v1 + v2));
}

// Pairs, final top-knn and softmax of one (token, head) row, given each half's top-knn keys (lane a holds
// entry a of the sorted lists, keys in the u64 format above). Writes row `row` of the outputs.
template <bool F32>
__device__ void cartesian_select(uint64_t key1, uint64_t key2, int nk, int knn, uint64_t* buf, uint32_t* sfix,
                                 int64_t row, void* scores_out, int64_t* idx_out, float* w_out) {
    const int lane = lane_id();
    const float v1 = score_of_code<F32>(key_code(key1));
    const float v2 = score_of_code<F32>(key_code(key2));
    const uint32_t i1 = key_index(key1), i2 = key_index(key2);

    // dominance-pruned pairs: lane a owns b < m_a = knn / (a + 1); at most 119 (knn = 32) pairs, held in
    // registers as candidate c = 32 r + lane, r < 4, and reduced to the sorted top 32 without shared memory
    const int m_a = lane < knn ? knn / (lane + 1) : 0;
    int incl = m_a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl += x;
    }
    const int total = __shfl_sync(FULL, incl, 31);
    const int off_a = incl - m_a;
    uint64_t cand[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int c = 32 * r + lane;
        // the row a of candidate c: the last a with off_a <= c (offsets ascend with a)
        int a = 0;
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
            const int probe = a + step;
            const int off_p = __shfl_sync(FULL, off_a, probe & 31);
            if (probe < 32 && off_p <= c) a = probe;
        }
        const int b = c - __shfl_sync(FULL, off_a, a);
        const float v1a = __shfl_sync(FULL, v1, a);
        const uint32_t i1a = __shfl_sync(FULL, i1, a);
        const float v2b = __shfl_sync(FULL, v2, b & 31);
        const uint32_t i2b = __shfl_sync(FULL, i2, b & 31);
        cand[r] = c < total ? make_key(pair_code<F32>(v1a, v2b), i1a * (uint32_t)nk + i2b) : 0;
    }
    const uint64_t best_all = warp_top32_of_128(cand, lane);
    const uint64_t best = lane < knn ? best_all : 0;
    const uint32_t t_code = key_code(__shfl_sync(FULL, best, knn - 1));

    // a pair outside the pruned set can only tie with T at the first excluded column of each list row
    bool tie_out = false;
    {
        const int bu = m_a < knn ? m_a : 0;
        const float v2u = __shfl_sync(FULL, v2, bu);
        tie_out = lane < knn && m_a < knn && pair_code<F32>(v1, v2u) == t_code;
    }
    uint64_t out_key = best;
    if (__ballot_sync(FULL, tie_out)) {
        const int c = __popc(__ballot_sync(FULL, lane < knn && key_code(best) > t_code));
        unsigned mask = 0;
        for (int b = 0; b < knn; b++) {
            const float v2b = __shfl_sync(FULL, v2, b);
            if (lane < knn && pair_code<F32>(v1, v2b) == t_code) mask |= 1u << b;
        }
        sfix[lane] = i2;
        __syncwarp();
        for (int r = c; r < knn; r++) {
            uint32_t mine = 0xffffffffu;
            for (unsigned mm = mask; mm; mm &= mm - 1) {
                const int b = __ffs(mm) - 1;
                const uint32_t full = i1 * (uint32_t)nk + sfix[b];
                mine = full < mine ? full : mine;
            }
            uint32_t win = mine;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) win = min(win, __shfl_xor_sync(FULL, win, o));
            if (mine == win && mask) {
                const uint32_t j2 = win - i1 * (uint32_t)nk;
                for (unsigned mm = mask; mm; mm &= mm - 1) {
                    const int b = __ffs(mm) - 1;
                    if (sfix[b] == j2) { mask &= ~(1u << b); break; }
                }
            }
            if (lane == r) out_key = make_key(t_code, win);
        }
        __syncwarp();
    }

    // softmax over the knn selected scores, fp32
    const float sc = score_of_code<F32>(key_code(out_key));
    const float mx = warp_max(lane < knn ? sc : -INFINITY);
    const float e = lane < knn ? expf(sc - mx) : 0.f;
    const float tot = warp_sum(e);
    if (lane < knn) {
        const int64_t o = row * knn + lane;
        if constexpr (F32) static_cast<float*>(scores_out)[o] = sc;
        else static_cast<uint16_t*>(scores_out)[o] = (uint16_t)decode_code16(key_code(out_key));
        idx_out[o] = key_index(out_key);
        w_out[o] = e / tot;
    }
    __syncwarp();
}

template <bool F32>
__global__ void __launch_bounds__(SEL_WARPS * 32) pk_select_kernel(const void* s1, const void* s2, int64_t rows_nh,
                                                                    int nk, int knn, void* scores_out,
                                                                    int64_t* idx_out, float* w_out) {
    __shared__ uint64_t sbuf[SEL_WARPS][SEL_CAP];
    __shared__ uint32_t sfix[SEL_WARPS][32];
    const int lane = lane_id();
    const int wib = threadIdx.x >> 5;
    uint64_t* buf = sbuf[wib];
    const int64_t warps = (int64_t)gridDim.x * SEL_WARPS;
    for (int64_t row = (int64_t)blockIdx.x * SEL_WARPS + wib; row < rows_nh; row += warps) {
        const int64_t off = row * nk;
        half_topk<F32>(s1, off, nk, knn, buf);
        const uint64_t key1 = lane < knn ? buf[lane] : 0;
        __syncwarp();
        half_topk<F32>(s2, off, nk, knn, buf);
        const uint64_t key2 = lane < knn ? buf[lane] : 0;
        __syncwarp();
        cartesian_select<F32>(key1, key2, nk, knn, buf, sfix[wib], row, scores_out, idx_out, w_out);
    }
}

constexpr int PAIR_BATCH = 16;  // top lists loaded together by the pair kernel

// Pairs + softmax from per-half top lists of bf16 scores, as written by the fused scoring kernel:
// lists[row][half][list] hold 32 keys (order code of the bf16 score << 16 | (0xffff - sub-key index)), sorted
// descending, one list per (key-range split, column set); the lists of a half are merged here.
__global__ void __launch_bounds__(SEL_WARPS * 32) pk_pairs_kernel(const uint32_t* lists, int lists_per_half,
                                                                   int64_t rows_nh, int nk, int knn,
                                                                   void* scores_out, int64_t* idx_out,
                                                                   float* w_out) {
    __shared__ uint64_t sbuf[SEL_WARPS][SEL_CAP];
    __shared__ uint32_t sfix[SEL_WARPS][32];
    const int lane = lane_id();
    const int wib = threadIdx.x >> 5;
    const int64_t warps = (int64_t)gridDim.x * SEL_WARPS;
    for (int64_t row = (int64_t)blockIdx.x * SEL_WARPS + wib; row < rows_nh; row += warps) {
        uint32_t hk[2];
#pragma unroll
        for (int half = 0; half < 2; half++) {
            // sorted list + next sorted list -> the bitonic max sequence -> one sorted list, across lanes
            // (with key-range splits: many lists, loaded PAIR_BATCH at a time so their loads overlap)
            const uint32_t* l = lists + ((row * 2 + half) * lists_per_half) * 32;
            uint32_t k = l[lane];
            for (int i0 = 1; i0 < lists_per_half; i0 += PAIR_BATCH) {
                uint32_t nxt[PAIR_BATCH];
#pragma unroll
                for (int u = 0; u < PAIR_BATCH; u++) nxt[u] = i0 + u < lists_per_half ? l[(i0 + u) * 32 + 31 - lane] : 0u;
#pragma unroll
                for (int u = 0; u < PAIR_BATCH; u++) {
                    if (i0 + u >= lists_per_half) break;
                    k = max(k, nxt[u]);
#pragma unroll
                    for (int j = 16; j > 0; j >>= 1) {
                        const uint32_t x = __shfl_xor_sync(FULL, k, j);
                        k = (lane & j) ? min(k, x) : max(k, x);
                    }
                }
            }
            hk[half] = k;
        }
        const uint64_t key1 = lane < knn ? make_key(hk[0] >> 16, 0xffffu - (hk[0] & 0xffffu)) : 0;
        const uint64_t key2 = lane < knn ? make_key(hk[1] >> 16, 0xffffu - (hk[1] & 0xffffu)) : 0;
        cartesian_select<false>(key1, key2, nk, knn, sbuf[wib], sfix[wib], row, scores_out, idx_out, w_out);
    }
}

int launch_pk_pairs(const uint32_t* lists, int lists_per_half, int64_t rows_nh, int nk, int knn, void* scores,
                    int64_t* idx, float* w, cudaStream_t st) {
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows_nh + SEL_WARPS - 1) / SEL_WARPS,
                                                                   (int64_t)sm_count() * 8));
    pk_pairs_kernel<<<blocks, SEL_WARPS * 32, 0, st>>>(lists, lists_per_half, rows_nh, nk, knn, scores, idx, w);
    SMLM_LAUNCHED("pk_pairs_kernel");
    return SMLM_OK;
}

// ------------------------------------------------------------------------------------ selection backward
// Per selected pair (one lane each, lane < knn) of one (token, head): dl = w (g_w - sum(w g_w)) + g_scores,
// ds = dl rounded to the score type, then per sub-key of each half the sum of ds over the pairs that use it, in
// selection order (fp32), kept by the lane of the sub-key's first occurrence. Invalid indices contribute nothing.
struct PairGrad {
    uint32_t a1, a2;  // the pair's sub-keys
    float s1, s2;     // per-sub-key sums (meaningful on the first occurrence)
    bool first1, first2;
};

template <bool F32>
__device__ __forceinline__ PairGrad pair_grad(const int64_t* idx, const float* w, const float* gw, const void* gs,
                                              int64_t row, int nk, int knn, int lane) {
    const int64_t o = row * knn + lane;
    const bool on = lane < knn;
    const float wj = on ? w[o] : 0.f;
    float dl = 0.f;
    if (gw) {
        const float g = on ? gw[o] : 0.f;
        const float dot = warp_sum(wj * g);
        dl = wj * (g - dot);
    }
    if (gs && on) {
        const float g2 = F32 ? static_cast<const float*>(gs)[o] : bf16_bits_to_f32(static_cast<const uint16_t*>(gs)[o]);
        dl = dl + g2;
    }
    int64_t full = on ? idx[o] : 0;
    if (full < 0 || full >= (int64_t)nk * nk) full = 0, dl = 0.f;
    const float ds = F32 ? dl : round_bf16(dl);
    PairGrad r;
    r.a1 = (uint32_t)(full / nk);
    r.a2 = (uint32_t)(full % nk);
    r.s1 = r.s2 = 0.f;
    r.first1 = r.first2 = on;
    for (int j = 0; j < knn; j++) {
        const uint32_t b1 = __shfl_sync(FULL, r.a1, j);
        const uint32_t b2 = __shfl_sync(FULL, r.a2, j);
        const float dj = __shfl_sync(FULL, ds, j);
        if (b1 == r.a1) {
            r.s1 = r.s1 + dj;
            if (j < lane) r.first1 = false;
        }
        if (b2 == r.a2) {
            r.s2 = r.s2 + dj;
            if (j < lane) r.first2 = false;
        }
    }
    return r;
}

template <bool F32>
__device__ __forceinline__ void store_grad(void* dst, int64_t i, float v) {
    if constexpr (F32) static_cast<float*>(dst)[i] = v;
    else static_cast<uint16_t*>(dst)[i] = (uint16_t)f32_to_bf16_bits(v);
}

// Dense form: ds1 / ds2 (n, h, nk) rows zeroed, then each sub-key's sum written by its first occurrence.
template <bool F32>
__global__ void __launch_bounds__(256) select_backward_kernel(const int64_t* idx, const float* w, const float* gw,
                                                              const void* gs, int64_t rows_nh, int nk, int knn,
                                                              void* ds1, void* ds2) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows_nh; row += warps) {
        const PairGrad g = pair_grad<F32>(idx, w, gw, gs, row, nk, knn, lane);
        const int64_t base = row * nk;
        for (int k = lane; k < nk; k += 32) {
            store_grad<F32>(ds1, base + k, 0.f);
            store_grad<F32>(ds2, base + k, 0.f);
        }
        __syncwarp();
        if (g.first1) store_grad<F32>(ds1, base + g.a1, g.s1);
        if (g.first2) store_grad<F32>(ds2, base + g.a2, g.s2);
        __syncwarp();
    }
}

// Sparse form: per (token, head, half) the knn selected sub-keys become the lookups of a value bag over the
// sub-key table viewed as (h * 2 * nk, half) rows: on a sub-key's first occurrence, row (head * 2 + half) * nk +
// sub-key with the sub-key's sum as weight; on later occurrences row -1, weight 0 (skipped by the bag). dq is
// that bag over the keys; dkeys is the bag's row-sparse backward with the query halves as the output gradient.
template <bool F32>
__global__ void __launch_bounds__(256) select_grad_entries_kernel(const int64_t* idx, const float* w, const float* gw,
                                                                  const void* gs, int64_t rows_nh, int heads, int nk,
                                                                  int knn, int64_t* entry_rows, void* entry_w) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows_nh; row += warps) {
        const PairGrad g = pair_grad<F32>(idx, w, gw, gs, row, nk, knn, lane);
        if (lane < knn) {
            const int hh = (int)(row % heads);
            const int64_t e1 = (row * 2 + 0) * knn + lane, e2 = (row * 2 + 1) * knn + lane;
            entry_rows[e1] = g.first1 ? (int64_t)(hh * 2 + 0) * nk + g.a1 : -1;
            entry_rows[e2] = g.first2 ? (int64_t)(hh * 2 + 1) * nk + g.a2 : -1;
            store_grad<F32>(entry_w, e1, g.first1 ? g.s1 : 0.f);
            store_grad<F32>(entry_w, e2, g.first2 ? g.s2 : 0.f);
        }
    }
}

// -------------------------------------------------------------------------------- exact fp32 sub-key scores
// s[n, h, j] = fmaf chain over t of q[n, h, hf * half + t] * keys[h, hf, j, t], t ascending from acc = 0.
// 64 x 64 output tile per block, 4 x 4 per thread, t staged through shared memory 32 at a time.
constexpr int SC_BM = 64, SC_BN = 64, SC_BK = 32;

__global__ void __launch_bounds__(256) subkey_scores_kernel(const float* q, const float* keys, int64_t n, int h,
                                                            int nk, int half, float* s1, float* s2) {
    __shared__ float As[SC_BK][SC_BM + 4];
    __shared__ float Bs[SC_BK][SC_BN + 4];
    const int hh = blockIdx.z >> 1, hf = blockIdx.z & 1;
    const int64_t m0 = (int64_t)blockIdx.y * SC_BM;
    const int j0 = blockIdx.x * SC_BN;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t qstride = (int64_t)h * 2 * half;
    const float* qa = q + (int64_t)hh * 2 * half + (int64_t)hf * half;
    const float* kb = keys + ((int64_t)hh * 2 + hf) * nk * half;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
    for (int t0 = 0; t0 < half; t0 += SC_BK) {
        for (int e = threadIdx.x; e < SC_BM * SC_BK; e += 256) {
            const int mm = e / SC_BK, tt = e % SC_BK;
            const int64_t gm = m0 + mm;
            As[tt][mm] = (gm < n && t0 + tt < half) ? qa[gm * qstride + t0 + tt] : 0.f;
        }
        for (int e = threadIdx.x; e < SC_BN * SC_BK; e += 256) {
            const int jj = e / SC_BK, tt = e % SC_BK;
            const int gj = j0 + jj;
            Bs[tt][jj] = (gj < nk && t0 + tt < half) ? kb[(int64_t)gj * half + t0 + tt] : 0.f;
        }
        __syncthreads();
        const int tmax = min(SC_BK, half - t0);
        for (int tt = 0; tt < tmax; tt++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = As[tt][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = Bs[tt][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
    float* out = hf ? s2 : s1;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int64_t gm = m0 + ty * 4 + i;
        if (gm >= n) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int gj = j0 + tx * 4 + j;
            if (gj < nk) out[(gm * h + hh) * nk + gj] = acc[i][j];
        }
    }
}

}  // namespace smlm

using namespace smlm;

extern "C" int smlm_pk_select(const void* s1, const void* s2, int score_dtype, int64_t n, int64_t h, int64_t nk,
                              int64_t knn, void* scores, int64_t* indices, float* weights, void* stream) {
    SMLM_CHECK_ARG(score_dtype == SMLM_F32 || score_dtype == SMLM_BF16, "pk_select: scores must be fp32 or bf16");
    SMLM_CHECK_ARG(n >= 0 && h > 0, "pk_select: bad n / heads");
    SMLM_CHECK_ARG(knn >= 1 && knn <= 32, "pk_select: knn must be in [1, 32], got %lld", (long long)knn);
    SMLM_CHECK_ARG(nk >= knn && nk <= 65536, "pk_select: need knn <= n_keys <= 65536, got n_keys=%lld",
                   (long long)nk);
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(s1 && s2 && scores && indices && weights, "pk_select: null pointer");
    const int64_t rows = n * h;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + SEL_WARPS - 1) / SEL_WARPS,
                                                                   (int64_t)sm_count() * 8));
    cudaStream_t st = as_stream(stream);
    if (score_dtype == SMLM_F32)
        pk_select_kernel<true><<<blocks, SEL_WARPS * 32, 0, st>>>(s1, s2, rows, (int)nk, (int)knn, scores, indices,
                                                                  weights);
    else
        pk_select_kernel<false><<<blocks, SEL_WARPS * 32, 0, st>>>(s1, s2, rows, (int)nk, (int)knn, scores, indices,
                                                                   weights);
    SMLM_LAUNCHED("pk_select_kernel");
    return SMLM_OK;
}

extern "C" int smlm_select_backward(const int64_t* indices, const float* weights, const float* grad_w,
                                    const void* grad_scores, int score_dtype, int64_t n, int64_t h, int64_t nk,
                                    int64_t knn, void* ds1, void* ds2, void* stream) {
    SMLM_CHECK_ARG(score_dtype == SMLM_F32 || score_dtype == SMLM_BF16, "select_backward: fp32 or bf16 only");
    SMLM_CHECK_ARG(n >= 0 && h > 0 && knn >= 1 && knn <= 32 && nk >= knn && nk <= 65536,
                   "select_backward: bad sizes");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(indices && weights && ds1 && ds2, "select_backward: null pointer");
    const int64_t rows = n * h;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 16));
    cudaStream_t st = as_stream(stream);
    if (score_dtype == SMLM_F32)
        select_backward_kernel<true><<<blocks, 256, 0, st>>>(indices, weights, grad_w, grad_scores, rows, (int)nk,
                                                             (int)knn, ds1, ds2);
    else
        select_backward_kernel<false><<<blocks, 256, 0, st>>>(indices, weights, grad_w, grad_scores, rows, (int)nk,
                                                              (int)knn, ds1, ds2);
    SMLM_LAUNCHED("select_backward_kernel");
    return SMLM_OK;
}

extern "C" int smlm_subkey_scores_f32(const float* q, const float* keys, int64_t n, int64_t h, int64_t nk,
                                      int64_t half, float* s1, float* s2, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && h > 0 && nk > 0 && half > 0, "subkey_scores_f32: bad sizes");
    SMLM_CHECK_ARG(h * 2 <= 65535 && nk < (1 << 30) && half < (1 << 20), "subkey_scores_f32: size too large");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(q && keys && s1 && s2, "subkey_scores_f32: null pointer");
    dim3 grid((unsigned)((nk + SC_BN - 1) / SC_BN), (unsigned)((n + SC_BM - 1) / SC_BM), (unsigned)(h * 2));
    SMLM_CHECK_ARG(grid.y <= 65535, "subkey_scores_f32: too many tokens for one call (%lld)", (long long)n);
    subkey_scores_kernel<<<grid, 256, 0, as_stream(stream)>>>(q, keys, n, (int)h, (int)nk, (int)half, s1, s2);
    SMLM_LAUNCHED("subkey_scores_kernel");
    return SMLM_OK;
}

extern "C" int smlm_select_grad_entries(const int64_t* indices, const float* weights, const float* grad_w,
                                        const void* grad_scores, int score_dtype, int64_t n, int64_t h, int64_t nk,
                                        int64_t knn, int64_t* entry_rows, void* entry_weights, void* stream) {
    SMLM_CHECK_ARG(score_dtype == SMLM_F32 || score_dtype == SMLM_BF16, "select_grad_entries: fp32 or bf16 only");
    SMLM_CHECK_ARG(n >= 0 && h > 0 && knn >= 1 && knn <= 32 && nk >= knn && nk <= 65536,
                   "select_grad_entries: bad sizes");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(indices && weights && entry_rows && entry_weights, "select_grad_entries: null pointer");
    const int64_t rows = n * h;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 16));
    cudaStream_t st = as_stream(stream);
    if (score_dtype == SMLM_F32)
        select_grad_entries_kernel<true><<<blocks, 256, 0, st>>>(indices, weights, grad_w, grad_scores, rows, (int)h,
                                                                 (int)nk, (int)knn, entry_rows, entry_weights);
    else
        select_grad_entries_kernel<false><<<blocks, 256, 0, st>>>(indices, weights, grad_w, grad_scores, rows, (int)h,
                                                                  (int)nk, (int)knn, entry_rows, entry_weights);
    SMLM_LAUNCHED("select_grad_entries_kernel");
    return SMLM_OK;
}
