// Fused sub-key scoring + per-half top-k on the 5th-generation tensor cores (sm_100a).
//
// For one head h and one half of the query (k = 128 dimensions), scores S = Q_h,half (tokens x 128) x K_h,half^T
// (128 x n_keys) are a bf16 GEMM with fp32 accumulation. S never reaches global memory: each accumulator tile
// lives in tensor memory (TMEM) and the epilogue keeps, per token, the top-32 of the bf16-rounded scores (order:
// score descending, sub-key index ascending), which is exactly what the reference's `einsum` (bf16 output) +
// per-half top-k computes. A second small kernel (select.cu, pk_pairs_kernel) forms the knn x knn pairs and the
// softmax from the two per-half lists.
//
// CTA = 10 warps, persistent over units (128-token tile, head, key-range split); a unit runs half 0 then half 1.
// With at least as many (tile, head) pairs as SMs there is one split (all key tiles); with fewer (decoding, short
// prompts) the key tiles are divided among up to #SMs / #pairs splits, each writing its own per-half top lists
// (a split of fewer than PRE_MIN_TILES key tiles skips the pre-pass described below):

//   warp 0      TMA producer: Q tile (128 tokens x 128, two 64-wide 128B-swizzled boxes) and key tiles
//               (128 keys x 128) through a 3-stage ring, completion by mbarrier transaction counts.
//   warp 1      allocates 256 TMEM columns (two 128-column fp32 accumulators); lane 0 issues tcgen05.mma
//               (M=128, N=128, K=16, kind::f16, bf16 in / fp32 accumulate), 8 per key tile, and commits to
//               the stage's "empty" barrier and the accumulator's "full" barrier.
//   warps 2-9   epilogue: tcgen05.ld of the 128 x 128 accumulator; warp w reads TMEM lanes 32 (w % 4) ..
//               (the lane quarter it may access), one token per thread, and columns [0, 64) (warps 2-5) or
//               [64, 128) (warps 6-9) of every tile.
// Each half's key tiles go through the tensor cores twice (the GEMM is cheap next to the selection). Pre-pass:
// every thread keeps the 32 largest maxima of its 32-column groups; their 32nd is a bf16 score that 32
// distinct columns reach, so the token's top 32 lies at or above it (the two column-set threads of a token
// take the larger of their two bounds). Selection pass: each score is compared in fp32 against the exact
// rounding bound of max(that floor, the thread's current 32nd-best); the few survivors queue in a per-thread
// list in shared memory, and once any lane holds FLUSH_AT of them the warp merges them in lockstep, 16 at a
// time (sort the batch, bitonic merge into the register-resident sorted top-32). Each token ends with one
// sorted top-32 per column set; the pair kernel merges the two.
// Every mbarrier wait is bounded (about one second); on timeout the kernel raises SMLM_FLAG_TIMEOUT in the
// status word, every role unwinds, the MMA issuer waits (bounded) for its last commit, and TMEM is freed.
// No TMA multicast is used (the kernel only reads this GPU's memory).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace smlm {

int launch_pk_pairs(const uint32_t* lists, int lists_per_half, int64_t rows_nh, int nk, int knn, void* scores,
                    int64_t* idx, float* w, cudaStream_t st);

namespace tc {

constexpr int BM = 128;          // tokens per tile (UMMA M)
constexpr int BN = 128;          // sub-keys per tile (UMMA N)
constexpr int STAGES = 3;        // key-tile ring
constexpr int EPI_WARPS = 8;     // two per TMEM lane quarter: column halves [0, 64) and [64, 128) of a tile
constexpr int EPI_THREADS = EPI_WARPS * 32;
constexpr int THREADS = 64 + EPI_THREADS;
constexpr int BATCH = 16;        // candidates merged into the top-32 per sorted batch
constexpr int FLUSH_AT = BATCH;  // a warp merges its candidates once any lane holds this many
constexpr int CAND = 48;         // >= FLUSH_AT - 1 + 32 (one chunk can add 32)
constexpr int ATOM = 64;         // bf16 elements per 128-byte swizzle atom (K direction)
constexpr int ATOM_BYTES_A = BM * 128;
constexpr int ATOM_BYTES_B = BN * 128;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr unsigned long long WAIT_NS = 1000000000ull;  // bound of every mbarrier wait
constexpr int PRE_MIN_TILES = 16;  // key tiles a unit needs before the pre-pass can yield a bound

// ------------------------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// The waiting thread may be suspended (up to ~0.1 ms) until the phase completes instead of spinning, so
// waiting warps leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}
// Bounded wait: false (and the abort flag set) if the phase did not complete within WAIT_NS or another role
// has aborted already.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (now_ns() - t0 > WAIT_NS) {
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

// Bounded wait that ignores the abort flag (used to drain in-flight MMAs before TMEM is freed).
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = now_ns();
    while (!mbar_try_wait(bar, parity) && now_ns() - t0 < WAIT_NS) {
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] x B[smem]^T, bf16 operands, fp32 accumulator.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes: thread t gets lane (base + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major, 128B-swizzled operand tile (rows of 128 bytes, 8-row groups
// 1024 bytes apart): start address >> 4, leading offset 1 (unused for this layout), stride offset 1024 >> 4,
// descriptor version 1, swizzle mode 2 (128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3ffffu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, N >> 3, M >> 4.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

// ------------------------------------------------------------------------------------------ top-k pieces
template <int N>
__device__ __forceinline__ void sort_desc(uint32_t (&a)[N]) {
#pragma unroll
    for (int k = 2; k <= N; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
            for (int i = 0; i < N; i++) {
                const int l = i ^ j;
                if (l > i) {
                    const uint32_t x = a[i], y = a[l];
                    const uint32_t hi = max(x, y), lo = min(x, y);
                    if ((i & k) == 0) { a[i] = hi; a[l] = lo; }
                    else { a[i] = lo; a[l] = hi; }
                }
            }
}

// a is bitonic; sorts it descending (5 stages of 16 independent compare-exchanges)
__device__ __forceinline__ void merge_desc32(uint32_t (&a)[32]) {
#pragma unroll
    for (int j = 16; j > 0; j >>= 1)
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int l = i ^ j;
            if (l > i) {
                const uint32_t x = a[i], y = a[l];
                a[i] = max(x, y);
                a[l] = min(x, y);
            }
        }
}

// key of a bf16 score: order code << 16 | (0xffff - sub-key index); larger is better, distinct per index
__device__ __forceinline__ uint32_t score_key(uint32_t bits16, int col) {
    return (order_code16(bits16) << 16) | (uint32_t)(0xffff - col);
}

// Smallest fp32 b such that bf16_rn(v) > t exactly when v >= b (t: bf16 bits of a finite threshold or -inf).
// With u the next bf16 above t, the rounding midpoint m = (t + u) / 2 rounds to the even one of t, u: it passes
// if u is even, otherwise only values above m pass.
__device__ __forceinline__ float pass_bound(uint32_t t) {
    uint32_t u;
    if ((t & 0x8000u) == 0) u = t + 1;           // +0 and positives: one step up
    else if (t == 0x8000u) u = 0x0001u;          // -0 -> smallest positive
    else u = t - 1;                              // negatives: one step toward zero
    const float m = 0.5f * (bf16_bits_to_f32(t) + bf16_bits_to_f32(u));  // exact
    if ((u & 1u) == 0) return m;
    const uint32_t mb = __float_as_uint(m);
    return __uint_as_float(m > 0.f ? mb + 1 : mb - 1);                   // next fp32 above m
}

// Smallest fp32 b such that bf16_rn(v) >= t exactly when v >= b: the pass bound of the next bf16 below t
// (+0 and -0 are one value; t = -inf lets everything pass).
__device__ __forceinline__ float pass_bound_ge(uint32_t t) {
    if (t == 0xff80u) return -INFINITY;
    uint32_t p;
    if (t == 0x0000u || t == 0x8000u) p = 0x8001u;   // just below zero: the negative subnormal closest to it
    else if (t & 0x8000u) p = t + 1;                   // negatives: one step away from zero
    else p = t - 1;                                    // positives: one step toward zero
    return pass_bound(p);
}

// The two column-set threads of a token (epilogue threads e and e ^ 128) swap their pre-pass bounds through
// shared memory: each publishes (sequence << 32) | bound and polls for the partner's entry of the same sequence,
// for a bounded time; if it does not come (an aborting partner), its own bound, equally valid, is used.
__device__ __forceinline__ uint32_t exchange_bound(uint64_t* pre, int e, uint32_t seq, uint32_t own,
                                                   volatile int* abort_flag) {
    volatile uint64_t* slots = pre;
    slots[e] = ((uint64_t)seq << 32) | own;
    __threadfence_block();
    const uint64_t t0 = now_ns();
    while (true) {
        const uint64_t p = slots[e ^ 128];
        if ((uint32_t)(p >> 32) == seq) return (uint32_t)p;
        if (*abort_flag || now_ns() - t0 > WAIT_NS) return own;
    }
}

// Per-thread (= per token) running top-32 of one column stream, in registers, sorted descending.
struct Epi {
    uint32_t* cand;   // [CAND][EPI_THREADS] candidate keys (slot-major: conflict-free per-thread lists)
    float4* stage;    // [8][EPI_THREADS] the chunk's 32 scores, for reading survivors back by index
    int e;            // epilogue thread index
    int cnt;
    uint32_t top[32];
    float bound;      // fp32 scores >= bound round to a bf16 above the current 32nd-best (and >= floor)
    float floor;      // scores below the token's pre-pass bound never enter the union's top 32

    __device__ __forceinline__ void set_thr() {
        bound = fmaxf(pass_bound(top[31] ? decode_code16(top[31] >> 16) : 0xff80u), floor);  // < 32 yet: -inf
    }
    // Pre-pass: the maximum of 32 consecutive scores (columns >= nk excluded) is queued as a key; the merged list
    // then holds the 32 largest such group maxima, and its 32nd entry is a score reached by 32 distinct columns.
    __device__ __forceinline__ void group_max(const uint32_t (&v)[32], int col0, int nk) {
        float mx;
        if (col0 + 32 <= nk) {  // warp-uniform: a full group, a plain max tree
            float m[16];
#pragma unroll
            for (int i = 0; i < 16; i++) m[i] = fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 16]));
#pragma unroll
            for (int w = 8; w > 0; w >>= 1)
#pragma unroll
                for (int i = 0; i < w; i++) m[i] = fmaxf(m[i], m[i + w]);
            mx = m[0];
        } else {
            float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < 32; i++)
                if (col0 + i < nk) m[i & 3] = fmaxf(m[i & 3], __uint_as_float(v[i]));
            mx = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
        }
        cand[cnt * EPI_THREADS + e] =
            mx == -INFINITY ? 0u : order_code16(__bfloat16_as_ushort(__float2bfloat16_rn(mx))) << 16;
        cnt++;
    }
    __device__ __forceinline__ void clear() {
#pragma unroll
        for (int i = 0; i < 32; i++) top[i] = 0u;
        cnt = 0;
    }
    // candidates [base, base + BATCH) enter the list: sort the batch, take the elementwise max of the list's tail
    // and the reversed batch (a bitonic sequence holding the best 32 of both), clean it into order
    __device__ __forceinline__ void merge_batch(int base) {
        uint32_t c[BATCH];
#pragma unroll
        for (int i = 0; i < BATCH; i++) c[i] = base + i < cnt ? cand[(base + i) * EPI_THREADS + e] : 0u;
        sort_desc<BATCH>(c);
#pragma unroll
        for (int i = 0; i < BATCH; i++) top[32 - BATCH + i] = max(top[32 - BATCH + i], c[BATCH - 1 - i]);
        merge_desc32(top);
    }
    __device__ __forceinline__ void dump(const uint32_t (&v)[32], int col0, int nk, uint16_t* dbg) {
        if (!dbg) return;
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (col0 + i < nk) dbg[col0 + i] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[i])));
    }
    // merges the buffered candidates, all lanes in lockstep, BATCH at a time
    __device__ __forceinline__ void flush() {
        const int mx = __reduce_max_sync(FULL, (unsigned)cnt);
        for (int base = 0; base < mx; base += BATCH) merge_batch(base);
        cnt = 0;
        set_thr();
    }
    // Pass 2 of a stream starts with an empty list and the floor from the pre-pass bound t (bf16 order code of
    // a score that 32 distinct columns of the token reach; 0: none): scores equal to it still pass.
    __device__ __forceinline__ void start_pass2(uint32_t t) {
        clear();
        floor = t ? pass_bound_ge(decode_code16(t)) : -INFINITY;
        set_thr();
    }
    // 32 consecutive scores (fp32 bits) of columns col0 .. col0+31: an fp32 compare against the exact bound
    // filters them; survivors are queued, and merged once any lane has FLUSH_AT of them.
    __device__ __forceinline__ void take(const uint32_t (&v)[32], int col0, int nk, uint16_t* dbg) {
        dump(v, col0, nk, dbg);
        uint32_t part[4] = {0u, 0u, 0u, 0u};  // four independent chains
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (__uint_as_float(v[i]) >= bound) part[i & 3] |= 1u << i;
        uint32_t bits = (part[0] | part[1]) | (part[2] | part[3]);
        if (col0 + 32 > nk) bits &= nk - col0 <= 0 ? 0u : (0xffffffffu >> (32 - (nk - col0)));
        if (bits) {
#pragma unroll
            for (int j = 0; j < 8; j++)
                stage[j * EPI_THREADS + e] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                         __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
            const float* sf = reinterpret_cast<const float*>(stage);
            while (bits) {
                const int i = __ffs(bits) - 1;
                bits &= bits - 1;
                const float x = sf[((i >> 2) * EPI_THREADS + e) * 4 + (i & 3)];
                cand[cnt * EPI_THREADS + e] = score_key(__bfloat16_as_ushort(__float2bfloat16_rn(x)), col0 + i);
                cnt++;
            }
        }
        if (__any_sync(FULL, cnt >= FLUSH_AT)) flush();
    }
};

struct Params {
    int n, heads, nk, atoms;  // atoms = half / 64
    int splits;               // key-range splits per (tile, head): 1, or more when there are few token tiles
    uint32_t* lists;          // [n][heads][2 halves][splits][2 column sets][32]
    uint16_t* dbg1;           // optional bf16 scores [n][heads][nk], half 0
    uint16_t* dbg2;           // half 1
    int* status;
};

__global__ void __launch_bounds__(THREADS, 1) score_topk_kernel(const __grid_constant__ CUtensorMap tq,
                                                                const __grid_constant__ CUtensorMap tk, Params P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int a_bytes = P.atoms * ATOM_BYTES_A;
    const int b_bytes = P.atoms * ATOM_BYTES_B;
    uint8_t* sA = smem;                              // a_bytes (one query tile)
    uint8_t* sB = sA + a_bytes;                      // STAGES x b_bytes
    uint32_t* cand = reinterpret_cast<uint32_t*>(sB + STAGES * b_bytes);
    float4* stage = reinterpret_cast<float4*>(cand + CAND * EPI_THREADS);
    uint64_t* pre = reinterpret_cast<uint64_t*>(stage + 8 * EPI_THREADS);  // [EPI_THREADS] pre-pass bounds
    uint64_t* bars = pre + EPI_THREADS;
    uint64_t* full_b = bars;
    uint64_t* empty_b = bars + STAGES;
    uint64_t* a_full = bars + 2 * STAGES;
    uint64_t* a_empty = a_full + 1;
    uint64_t* t_full = a_empty + 1;
    uint64_t* t_empty = t_full + 2;
    uint64_t* done = t_empty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (P.n + BM - 1) / BM;
    const int units = tiles_m * P.heads * P.splits;
    const int ntiles = (P.nk + BN - 1) / BN;
    // unit u = ((tile * heads) + head) * splits + split; split s covers key tiles [kt0, kt1)
    auto unit_tiles = [&](int u, int& kt0) {
        const int s = u % P.splits;
        kt0 = (int)((int64_t)s * ntiles / P.splits);
        return (int)((int64_t)(s + 1) * ntiles / P.splits) - kt0;
    };
    // passes over a unit's key tiles: the pre-pass only yields a bound once a thread holds 32 group maxima (two
    // per tile), so units of fewer than PRE_MIN_TILES tiles go straight to the selection pass
    auto unit_passes = [](int nt) { return nt >= PRE_MIN_TILES ? 2 : 1; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(smem_addr(&full_b[i]), 1);
            mbar_init(smem_addr(&empty_b[i]), 1);
        }
        mbar_init(smem_addr(a_full), 1);
        mbar_init(smem_addr(a_empty), 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_addr(&t_full[i]), 1);
            mbar_init(smem_addr(&t_empty[i]), EPI_WARPS);
        }
        mbar_init(smem_addr(done), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_holder), TMEM_COLS);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < EPI_THREADS; i += THREADS) pre[i] = 0;  // sequence 0: nothing published
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int a_iter = 0;
            for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
                const int tm = u / P.splits / P.heads, h = (u / P.splits) % P.heads;
                int kt0;
                const int nt = unit_tiles(u, kt0);
                const int np = unit_passes(nt);
                for (int half = 0; half < 2; half++) {
                    if (!mbar_wait(smem_addr(a_empty), (a_iter & 1) ^ 1, abort_flag)) break;
                    mbar_expect_tx(smem_addr(a_full), a_bytes);
                    for (int i = 0; i < P.atoms; i++)
                        tma_load_3d(smem_addr(sA + i * ATOM_BYTES_A), &tq, smem_addr(a_full), i * ATOM, h * 2 + half,
                                    tm * BM);
                    a_iter++;
                    for (int t = 0; t < np * nt; t++) {  // (pre-pass, then) the selection pass
                        const int kt = kt0 + (t < nt ? t : t - nt);
                        if (!mbar_wait(smem_addr(&empty_b[s]), ph ^ 1, abort_flag)) break;
                        mbar_expect_tx(smem_addr(&full_b[s]), b_bytes);
                        for (int i = 0; i < P.atoms; i++)
                            tma_load_2d(smem_addr(sB + s * b_bytes + i * ATOM_BYTES_B), &tk, smem_addr(&full_b[s]),
                                        i * ATOM, (h * 2 + half) * P.nk + kt * BN);
                        if (++s == STAGES) { s = 0; ph ^= 1; }
                    }
                    if (*abort_flag) break;
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int a_iter = 0, t_iter = 0;
            for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
                int kt0;
                const int nt = unit_tiles(u, kt0);
                const int np = unit_passes(nt);
                for (int half = 0; half < 2; half++) {
                    if (!mbar_wait(smem_addr(a_full), a_iter & 1, abort_flag)) break;
                    fence_after();
                    const uint32_t a_base = smem_addr(sA);
                    for (int t = 0; t < np * nt; t++) {  // the key tiles once per pass (pre-pass, selection)
                        if (!mbar_wait(smem_addr(&full_b[s]), ph, abort_flag)) break;
                        const int tb = t_iter & 1;
                        if (!mbar_wait(smem_addr(&t_empty[tb]), ((t_iter >> 1) & 1) ^ 1, abort_flag)) break;
                        fence_after();
                        const uint32_t d = tmem + tb * BN;
                        const uint32_t b_base = smem_addr(sB + s * b_bytes);
                        for (int i = 0; i < P.atoms; i++) {
#pragma unroll
                            for (int j = 0; j < ATOM / 16; j++) {
                                const uint64_t ad = sw128_desc(a_base + i * ATOM_BYTES_A + j * 32);
                                const uint64_t bd = sw128_desc(b_base + i * ATOM_BYTES_B + j * 32);
                                umma_bf16(d, ad, bd, IDESC, (i | j) != 0);
                            }
                        }
                        umma_commit(smem_addr(&empty_b[s]));
                        umma_commit(smem_addr(&t_full[tb]));
                        t_iter++;
                        if (++s == STAGES) { s = 0; ph ^= 1; }
                    }
                    umma_commit(smem_addr(a_empty));
                    a_iter++;
                    if (*abort_flag) break;
                }
            }
            // all issued MMAs complete before TMEM can be freed
            umma_commit(smem_addr(done));
            mbar_wait_drain(smem_addr(done), 0);
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int quarter = warp & 3;           // TMEM lane quarter this warp may access
        const int cset = (warp - 2) >> 2;        // column set: [0, 64) or [64, 128) of every tile
        const int row = quarter * 32 + lane;    // token row within the tile
        Epi ep;
        ep.cand = cand;
        ep.stage = stage;
        ep.e = (warp - 2) * 32 + lane;
        ep.cnt = 0;
        int t_iter = 0;
        uint32_t pre_seq = 0;
        for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
            const int tm = u / P.splits / P.heads, h = (u / P.splits) % P.heads, split = u % P.splits;
            int kt0;
            const int nt = unit_tiles(u, kt0);
            const int np = unit_passes(nt);
            const int64_t n = (int64_t)tm * BM + row;
            for (int half = 0; half < 2; half++) {
                uint16_t* dbg = half ? P.dbg2 : P.dbg1;
                if (dbg && n < P.n) dbg += (n * P.heads + h) * (int64_t)P.nk;
                else dbg = nullptr;
                bool ok = true;
                ep.clear();
                ep.floor = -INFINITY;
                if (np == 1) ep.start_pass2(0u);
                for (int t = 0; t < np * nt; t++) {
                    const int tb = t_iter & 1;
                    // warp-uniform outcome: the TMEM loads below are .sync.aligned
                    if (!__all_sync(FULL, mbar_wait(smem_addr(&t_full[tb]), (t_iter >> 1) & 1, abort_flag))) {
                        ok = false;
                        break;
                    }
                    fence_after();
                    const uint32_t base = tmem + ((uint32_t)(quarter * 32) << 16) + tb * BN + cset * 64;
                    uint32_t v0[32], v1[32];
                    tmem_ld32(base + 0, v0);
                    tmem_ld32(base + 32, v1);
                    tmem_wait_ld();
                    fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_addr(&t_empty[tb]));
                    t_iter++;
                    if (np == 2 && t < nt) {
                        // pre-pass: group maxima of 32 columns, merged 16 at a time (every lane holds the same count)
                        const int c0 = (kt0 + t) * BN + cset * 64;
                        ep.group_max(v0, c0, P.nk);
                        ep.group_max(v1, c0 + 32, P.nk);
                        if (ep.cnt == BATCH) ep.flush();
                        if (t == nt - 1) {
                            if (ep.cnt) ep.flush();
                            // the better of the two column-set threads' bounds (both are valid for the union)
                            const uint32_t own = ep.top[31] >> 16;
                            const uint32_t other = exchange_bound(pre, ep.e, ++pre_seq, own, abort_flag);
                            ep.start_pass2(max(own, other));
                        }
                    } else {
                        const int c0 = (kt0 + t - (np - 1) * nt) * BN + cset * 64;
                        ep.take(v0, c0, P.nk, dbg);
                        ep.take(v1, c0 + 32, P.nk, dbg);
                    }
                }
                if (!ok) break;
                if (__any_sync(FULL, ep.cnt > 0)) ep.flush();
                if (n < P.n) {
                    uint32_t* dst = P.lists + ((((n * P.heads + h) * 2 + half) * P.splits + split) * 2 + cset) * 32;
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<uint4*>(dst + i) = make_uint4(ep.top[i], ep.top[i + 1], ep.top[i + 2], ep.top[i + 3]);
                }
            }
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) flag(P.status, SMLM_FLAG_TIMEOUT);
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

size_t smem_bytes(int atoms) {
    return 1024 + (size_t)atoms * ATOM_BYTES_A + STAGES * (size_t)atoms * ATOM_BYTES_B + CAND * EPI_THREADS * 4 +
           8 * EPI_THREADS * 16 + EPI_THREADS * 8 + 16 * 8 + 16;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Key-range splits per (token tile, head): with fewer (tile, head) units than SMs (decoding, short prefills) each
// unit's key tiles are split over several CTAs, every split keeping its own per-half top lists, which the pair
// kernel merges (exact: each list is the top of its keys, and the top knn of all keys lies in their union).
// ntiles = 0: the upper bound over all key counts (what the workspace query sizes for).
int score_splits(int64_t n, int64_t h, int64_t ntiles) {
    const int64_t base = ((n + BM - 1) / BM) * h;
    int64_t s = base >= sm_count() ? 1 : std::max<int64_t>(1, sm_count() / std::max<int64_t>(base, 1));
    if (ntiles > 0) s = std::min(s, ntiles);
    return (int)std::max<int64_t>(1, std::min<int64_t>(s, 512));
}

// ------------------------------------------------------------------------------ few tokens: SIMT scoring
// Decoding and other calls of a few tokens have too little GEMM work to fill the tensor-core pipeline: the
// tcgen05 kernel then runs a few units split over the key range, each a chain of barrier set-up, TMEM allocation,
// TMA loads, one MMA per key tile and the merges, and the chain's latency is the call's time. For such calls each
// CTA instead scores SMALL_KEYS consecutive sub-keys of both halves of one (token, head) with plain FMAs (one
// sub-key per thread: its row read with 16-byte loads, an fp32 fmaf chain over the half dimension against the
// query half in shared memory, rounded once to bf16, as the reference's autocast einsum rounds its fp32
// accumulation), keeps the top 32 of each half (a warp sort per 32 sub-keys, then bitonic merges), and writes one
// list per half in the fused kernel's list format; the pair kernel merges the key ranges' lists as it merges the
// fused kernel's splits. Scores equal the fused kernel's wherever the two fp32 sums round to the same bf16 value
// (the order of fp32 additions differs; both are within one bf16 step of cuBLAS's einsum).
constexpr int SMALL_KEYS = 256;       // sub-keys per half per CTA (one per thread)
constexpr int SMALL_MAX_TOKENS = 16;  // calls of at most this many tokens take the SIMT path
constexpr int SMALL_MAX_RANGES = 32;  // key ranges per (token, head), so n_keys <= 8192

// Key ranges of the SIMT path for this call, 0 when the call takes the tensor-core kernel.
int small_ranges(int64_t n, int64_t nk) {
    if (n > SMALL_MAX_TOKENS || nk % SMALL_KEYS != 0 || nk / SMALL_KEYS > SMALL_MAX_RANGES) return 0;
    return (int)(nk / SMALL_KEYS);
}

__device__ __forceinline__ uint32_t warp_sort32_desc_u32(uint32_t v, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
        const bool desc = (lane & k) == 0;
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint32_t x = __shfl_xor_sync(FULL, v, j);
            v = (((lane & j) == 0) == desc) ? max(v, x) : min(v, x);
        }
    }
    return v;
}

// grid: n * h * ranges CTAs of SMALL_KEYS threads; lists[((row * 2 + half) * ranges + range) * 32 + i], row = t * h + hd
template <int HALF>
__global__ void __launch_bounds__(SMALL_KEYS) score_small_kernel(const uint16_t* q, const uint16_t* keys, int h,
                                                                 int nk, int ranges, uint32_t* lists, uint16_t* dbg1,
                                                                 uint16_t* dbg2) {
    constexpr int WARPS = SMALL_KEYS / 32;
    constexpr int VECS = HALF / 8;  // 16-byte vectors of 8 bf16 per sub-key row
    __shared__ float sq[2 * HALF];
    __shared__ uint32_t swl[WARPS][32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int range = (int)(blockIdx.x % ranges);
    const int64_t row = blockIdx.x / ranges;  // token * h + head
    const int hd = (int)(row % h);
    for (int i = tid; i < 2 * HALF; i += SMALL_KEYS) sq[i] = bf16_bits_to_f32(q[row * 2 * HALF + i]);
    __syncthreads();
    const int col = range * SMALL_KEYS + tid;
#pragma unroll 1
    for (int half = 0; half < 2; half++) {
        const uint4* krow = reinterpret_cast<const uint4*>(keys + ((int64_t)(hd * 2 + half) * nk + col) * HALF);
        uint4 kv[VECS];
#pragma unroll
        for (int i = 0; i < VECS; i++) kv[i] = __ldg(krow + i);
        const float* qh = sq + half * HALF;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < VECS; i++) {
            const uint32_t w4[4] = {kv[i].x, kv[i].y, kv[i].z, kv[i].w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                acc = fmaf(qh[8 * i + 2 * j], bf16_bits_to_f32(w4[j] & 0xffffu), acc);
                acc = fmaf(qh[8 * i + 2 * j + 1], bf16_bits_to_f32(w4[j] >> 16), acc);
            }
        }
        const uint32_t bits = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
        uint16_t* dbg = half ? dbg2 : dbg1;
        if (dbg) dbg[row * nk + col] = (uint16_t)bits;
        const uint32_t key = score_key(bits, col);
        swl[warp][lane] = warp_sort32_desc_u32(key, lane);
        __syncthreads();
        if (warp == 0) {
            // sorted list + reversed next sorted list -> their elementwise maxima hold the top 32 of both as a
            // bitonic sequence -> half-cleaners sort it
            uint32_t k = swl[0][lane];
#pragma unroll
            for (int w = 1; w < WARPS; w++) {
                k = max(k, swl[w][31 - lane]);
#pragma unroll
                for (int j = 16; j > 0; j >>= 1) {
                    const uint32_t x = __shfl_xor_sync(FULL, k, j);
                    k = (lane & j) ? min(k, x) : max(k, x);
                }
            }
            lists[((row * 2 + half) * ranges + range) * 32 + lane] = k;
        }
        __syncthreads();
    }
}

int launch_score_small(const void* q, const void* keys, int64_t n, int64_t h, int64_t nk, int64_t half, int ranges,
                       uint32_t* lists, void* s1_out, void* s2_out, cudaStream_t st) {
    const int64_t grid = n * h * ranges;
    auto* qq = static_cast<const uint16_t*>(q);
    auto* kk = static_cast<const uint16_t*>(keys);
    auto* d1 = static_cast<uint16_t*>(s1_out);
    auto* d2 = static_cast<uint16_t*>(s2_out);
    if (half == 128) score_small_kernel<128><<<(unsigned)grid, SMALL_KEYS, 0, st>>>(qq, kk, (int)h, (int)nk, ranges, lists, d1, d2);
    else score_small_kernel<64><<<(unsigned)grid, SMALL_KEYS, 0, st>>>(qq, kk, (int)h, (int)nk, ranges, lists, d1, d2);
    SMLM_LAUNCHED("score_small_kernel");
    return SMLM_OK;
}

}  // namespace tc
}  // namespace smlm

using namespace smlm;

extern "C" size_t smlm_score_select_workspace(int64_t n, int64_t h) {
    n = std::max<int64_t>(n, 0);
    h = std::max<int64_t>(h, 0);
    return (size_t)n * h * 2 * tc::score_splits(n, std::max<int64_t>(h, 1), 0) * 2 * 32 * sizeof(uint32_t) + 256;
}

extern "C" int smlm_score_select(const void* q, const void* keys, int64_t n, int64_t h, int64_t nk, int64_t half,
                                 int64_t knn, void* scores, int64_t* indices, float* weights, void* s1_out,
                                 void* s2_out, void* workspace, size_t workspace_bytes, int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && h > 0, "score_select: bad n / heads");
    SMLM_CHECK_ARG(half == 64 || half == 128, "score_select: the half dimension must be 64 or 128, got %lld",
                   (long long)half);
    SMLM_CHECK_ARG(knn >= 1 && knn <= 32, "score_select: knn must be in [1, 32]");
    SMLM_CHECK_ARG(nk >= knn && nk <= 65536 && nk % 8 == 0, "score_select: need knn <= n_keys <= 65536, n_keys % 8 == 0");
    SMLM_CHECK_ARG(n < (1ll << 31) / std::max<int64_t>(h, 1) / 64 && h * 2 * nk < (1ll << 31),
                   "score_select: sizes beyond 32-bit TMA coordinates");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(q && keys && scores && indices && weights, "score_select: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(keys) % 16 == 0,
                   "score_select: q and keys must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    const int ranges = tc::small_ranges(n, nk);
    if (ranges > 0 && workspace != nullptr &&
        workspace_bytes >= (size_t)n * h * 2 * ranges * 32 * sizeof(uint32_t)) {
        uint32_t* lists = static_cast<uint32_t*>(workspace);
        const int rc = tc::launch_score_small(q, keys, n, h, nk, half, ranges, lists, s1_out, s2_out, st);
        if (rc != SMLM_OK) return rc;
        return launch_pk_pairs(lists, ranges, n * h, (int)nk, (int)knn, scores, indices, weights, st);
    }
    const int splits = tc::score_splits(n, h, (nk + tc::BN - 1) / tc::BN);
    const size_t need = (size_t)n * h * 2 * splits * 2 * 32 * sizeof(uint32_t);
    if (workspace == nullptr || workspace_bytes < need) {
        set_error("score_select: workspace too small (%zu < %zu)", workspace_bytes, need);
        return SMLM_ERR_WORKSPACE;
    }
    auto encode = tc::encode_fn();
    if (!encode) {
        set_error("score_select: cuTensorMapEncodeTiled is not available from the driver");
        return SMLM_ERR_CUDA;
    }
    CUtensorMap tq, tk;
    {
        cuuint64_t dims[3] = {(cuuint64_t)half, (cuuint64_t)(2 * h), (cuuint64_t)n};
        cuuint64_t strides[2] = {(cuuint64_t)half * 2, (cuuint64_t)(2 * h * half * 2)};
        cuuint32_t box[3] = {tc::ATOM, 1, tc::BM};
        cuuint32_t es[3] = {1, 1, 1};
        CUresult r = encode(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, es,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            set_error("score_select: query tensor map encode failed (%d)", (int)r);
            return SMLM_ERR_CUDA;
        }
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)half, (cuuint64_t)(h * 2 * nk)};
        cuuint64_t strides[1] = {(cuuint64_t)half * 2};
        cuuint32_t box[2] = {tc::ATOM, tc::BN};
        cuuint32_t es[2] = {1, 1};
        CUresult r = encode(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(keys), dims, strides, box, es,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            set_error("score_select: key tensor map encode failed (%d)", (int)r);
            return SMLM_ERR_CUDA;
        }
    }
    uint32_t* lists = static_cast<uint32_t*>(workspace);
    const int atoms = (int)(half / tc::ATOM);
    const size_t smem = tc::smem_bytes(atoms);
    SMLM_CUDA(cudaFuncSetAttribute(tc::score_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t units = ((n + tc::BM - 1) / tc::BM) * h * splits;
    const int grid = (int)std::min<int64_t>(units, sm_count());
    tc::Params P{(int)n, (int)h, (int)nk, atoms, splits, lists, static_cast<uint16_t*>(s1_out),
                 static_cast<uint16_t*>(s2_out), status};
    tc::score_topk_kernel<<<grid, tc::THREADS, smem, st>>>(tq, tk, P);
    SMLM_LAUNCHED("score_topk_kernel");
    return launch_pk_pairs(lists, 2 * splits, n * h, (int)nk, (int)knn, scores, indices, weights, st);
}

// ------------------------------------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory at call time: a host framework that has reserved the GPU's memory
// in its own pool (so a cudaMalloc of the scratch would fail or fragment it), or a latency-critical serving
// loop where a cudaMalloc / cudaFree would synchronise the device. smlm_score_select_noalloc serves them: its
// scratch, the per-half top lists of at most SMLM_NOALLOC_MAX_ROWS (token, head) rows (512 bytes each, 8 MiB in
// all), is this array in the library's static device memory. Every GPU that loads the library holds it until
// the process exits. All calls share it, so calls that overlap on the GPU (other streams, other threads) race.
static __device__ __align__(256) uint32_t g_noalloc_lists[(size_t)SMLM_NOALLOC_MAX_ROWS * 2 * 2 * 32];

namespace smlm {
namespace tc {

// Device address of g_noalloc_lists on the current device, looked up once per device (host code only sees a
// host-side stand-in under that name, which must never reach a kernel).
static int noalloc_scratch(cudaStream_t stream, uint32_t** out) {
    static std::mutex mu;
    static uint32_t* addr[64] = {};
    int dev = 0;
    SMLM_CUDA(cudaGetDevice(&dev));
    SMLM_CHECK_ARG(dev >= 0 && dev < 64, "score_select_noalloc: device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        // the lookup may load the module, which a capturing stream does not allow: say so instead of failing
        // with a bare CUDA error
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        SMLM_CUDA(cudaStreamIsCapturing(stream, &cap));
        SMLM_CHECK_ARG(cap == cudaStreamCaptureStatusNone,
                       "score_select_noalloc: the first call on device %d must come before any stream capture "
                       "(it looks up the static scratch's device address)", dev);
        void* p = nullptr;
        SMLM_CUDA(cudaGetSymbolAddress(&p, g_noalloc_lists));
        addr[dev] = static_cast<uint32_t*>(p);
    }
    *out = addr[dev];
    return SMLM_OK;
}

}  // namespace tc
}  // namespace smlm

extern "C" int smlm_score_select_noalloc(const void* q, const void* keys, int64_t n, int64_t h, int64_t nk,
                                         int64_t half, int64_t knn, void* scores, int64_t* indices, float* weights,
                                         int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && h > 0, "score_select_noalloc: bad n / heads");
    // compared without forming n * h, which could wrap for absurd n
    SMLM_CHECK_ARG(n <= SMLM_NOALLOC_MAX_ROWS / h,
                   "score_select_noalloc: n = %lld tokens x %lld heads exceeds the static scratch "
                   "(SMLM_NOALLOC_MAX_ROWS = %d rows); split the call or use smlm_score_select with a workspace",
                   (long long)n, (long long)h, SMLM_NOALLOC_MAX_ROWS);
    SMLM_CHECK_ARG(half == 64 || half == 128, "score_select_noalloc: the half dimension must be 64 or 128, got %lld",
                   (long long)half);
    SMLM_CHECK_ARG(knn >= 1 && knn <= 32, "score_select_noalloc: knn must be in [1, 32]");
    SMLM_CHECK_ARG(nk >= knn && nk <= 65536 && nk % 8 == 0,
                   "score_select_noalloc: need knn <= n_keys <= 65536, n_keys % 8 == 0");
    SMLM_CHECK_ARG(h * 2 * nk < (1ll << 31), "score_select_noalloc: sizes beyond 32-bit TMA coordinates");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(q && keys && scores && indices && weights, "score_select_noalloc: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(keys) % 16 == 0,
                   "score_select_noalloc: q and keys must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    uint32_t* lists = nullptr;
    int rc = tc::noalloc_scratch(st, &lists);
    if (rc != SMLM_OK) return rc;
    // the workspace entry point's few-token path, whose lists (n * h * 2 * ranges * 32) fit the static array
    // whenever n is within its token limit
    const int ranges = tc::small_ranges(n, nk);
    if (ranges > 0 && n * h * ranges <= 2 * (int64_t)SMLM_NOALLOC_MAX_ROWS) {
        rc = tc::launch_score_small(q, keys, n, h, nk, half, ranges, lists, nullptr, nullptr, st);
        if (rc != SMLM_OK) return rc;
        return launch_pk_pairs(lists, ranges, n * h, (int)nk, (int)knn, scores, indices, weights, st);
    }
    auto encode = tc::encode_fn();
    if (!encode) {
        set_error("score_select_noalloc: cuTensorMapEncodeTiled is not available from the driver");
        return SMLM_ERR_CUDA;
    }
    CUtensorMap tq, tk;
    {
        cuuint64_t dims[3] = {(cuuint64_t)half, (cuuint64_t)(2 * h), (cuuint64_t)n};
        cuuint64_t strides[2] = {(cuuint64_t)half * 2, (cuuint64_t)(2 * h * half * 2)};
        cuuint32_t box[3] = {tc::ATOM, 1, tc::BM};
        cuuint32_t es[3] = {1, 1, 1};
        if (encode(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            set_error("score_select_noalloc: query tensor map encode failed");
            return SMLM_ERR_CUDA;
        }
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)half, (cuuint64_t)(h * 2 * nk)};
        cuuint64_t strides[1] = {(cuuint64_t)half * 2};
        cuuint32_t box[2] = {tc::ATOM, tc::BN};
        cuuint32_t es[2] = {1, 1};
        if (encode(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(keys), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            set_error("score_select_noalloc: key tensor map encode failed");
            return SMLM_ERR_CUDA;
        }
    }
    const int atoms = (int)(half / tc::ATOM);
    const size_t smem = tc::smem_bytes(atoms);
    SMLM_CUDA(cudaFuncSetAttribute(tc::score_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // key-range splits as the workspace entry point chooses them, as far as the static lists hold them (each
    // split keeps its own lists per row): small calls, decoding among them, still spread over the SMs
    const int splits = (int)std::max<int64_t>(
        1, std::min<int64_t>(tc::score_splits(n, h, (nk + tc::BN - 1) / tc::BN), SMLM_NOALLOC_MAX_ROWS / (n * h)));
    const int64_t units = ((n + tc::BM - 1) / tc::BM) * h * splits;
    const int grid = (int)std::min<int64_t>(units, sm_count());
    // every (token, head, split) row of the lists is written by the scoring kernel before the pair kernel reads
    // it, so the previous call's contents need no clearing
    tc::Params P{(int)n, (int)h, (int)nk, atoms, splits, lists, nullptr, nullptr, status};
    tc::score_topk_kernel<<<grid, tc::THREADS, smem, st>>>(tq, tk, P);
    SMLM_LAUNCHED("score_topk_kernel");
    return launch_pk_pairs(lists, 2 * splits, n * h, (int)nk, (int)knn, scores, indices, weights, st);
}
