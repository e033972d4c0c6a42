// Weighted value bag: forward gather, inference bag (fp32 / bf16 / q4 table, fused swilu), q4 quantisation,
// and the row-sparse backward (stable radix sort of (row, position) + deterministic segment sums).
//
// Layout: table (rows, d) row-major; indices / weights (n, k) row-major; one warp per (token, column block).
// Row loads are 16-byte (fp32) or 8-byte (bf16) vectors, one vector per lane per slot, so a warp reads a
// contiguous 512 B / 256 B stretch of a row per instruction.
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"

namespace smlm {

// ------------------------------------------------------------------------------------------- vector loads
__device__ __forceinline__ float load_weight(const void* w, int dtype, int64_t i) {
    if (dtype == SMLM_F32) return __ldg(static_cast<const float*>(w) + i);
    return bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(w) + i));
}

template <int VEC>
__device__ __forceinline__ void store_out(void* out, int dtype, int64_t off, const float (&v)[VEC]) {
    if (dtype == SMLM_F32) {
        float* o = static_cast<float*>(out) + off;
        if constexpr (VEC == 4) {
            *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; i++) o[i] = v[i];
        }
    } else {
        uint16_t* o = static_cast<uint16_t*>(out) + off;
#pragma unroll
        for (int i = 0; i < VEC; i++) o[i] = (uint16_t)f32_to_bf16_bits(v[i]);
    }
}


// ---------------------------------------------------------------------------------------------- bag gather
// Lookup indices: int64 or int32 global rows; the table holds rows [row_base, row_base + rows). Rows outside
// that range are skipped: flagged as an index error, or silently when skip_foreign (a row shard, whose other
// rows live on other GPUs).
__device__ __forceinline__ int64_t load_index(const void* idx, int idx32, int64_t i) {
    return idx32 ? (int64_t)__ldg(static_cast<const int32_t*>(idx) + i) : __ldg(static_cast<const int64_t*>(idx) + i);
}

struct BagArgs {
    const void* idx;
    int idx32;
    int64_t row_base;
    int skip_foreign;
    const void* w;
    int w_dtype;
    const void* table;
    const void* pre;  // swilu pre-activation or NULL
    int pre_dtype;
    void* out;
    int out_dtype;
    int64_t n, rows;
    int k, d;
    int col_block;  // columns per warp task = 32 * VEC * NS
    int* status;
};

// One warp per (token, column block); j-loop over the token's k lookups in chunks of 32 (lane j holds the
// j-th index / weight of the chunk). The chunk's valid lookups (a warp ballot, in j order) are taken four at a
// time, four rows in flight per step. The accumulation is a sequential fmaf chain over the valid j for every
// column.
template <typename TT, int VEC, int NS>
__global__ void __launch_bounds__(256) bag_gather_kernel(BagArgs a) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int nblk = (a.d + a.col_block - 1) / a.col_block;
    const TT* table = static_cast<const TT*>(a.table);
    for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < a.n * nblk;
         task += warps) {
        const int64_t n = task / nblk;
        const int c0 = (int)(task % nblk) * a.col_block;
        float acc[NS][VEC];
#pragma unroll
        for (int s = 0; s < NS; s++)
#pragma unroll
            for (int i = 0; i < VEC; i++) acc[s][i] = 0.f;
        for (int j0 = 0; j0 < a.k; j0 += 32) {
            const int cnt = min(32, a.k - j0);
            int64_t my_r = -1;
            float my_w = 0.f;
            if (lane < cnt) {
                my_r = load_index(a.idx, a.idx32, n * a.k + j0 + lane) - a.row_base;
                my_w = load_weight(a.w, a.w_dtype, n * a.k + j0 + lane);
                if (my_r < 0 || my_r >= a.rows) {
                    if (!a.skip_foreign) flag(a.status, SMLM_FLAG_INDEX_RANGE);
                    my_r = -1;
                }
            }
            unsigned todo = __ballot_sync(FULL, my_r >= 0);
            while (todo) {  // warp-uniform
                int64_t r[4];
                float wv[4];
                bool ok[4];
                float v[4][NS][VEC];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    ok[u] = todo != 0;
                    const int src = ok[u] ? __ffs(todo) - 1 : 0;
                    todo &= todo - 1;
                    r[u] = __shfl_sync(FULL, my_r, src);
                    wv[u] = __shfl_sync(FULL, my_w, src);
#pragma unroll
                    for (int s = 0; s < NS; s++) {
                        const int col = c0 + (lane + 32 * s) * VEC;
                        if (ok[u] && col < a.d) {
                            Elt<TT>::template load<VEC>(table + r[u] * a.d + col, v[u][s]);
                        } else {
#pragma unroll
                            for (int i = 0; i < VEC; i++) v[u][s][i] = 0.f;
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; u++)
#pragma unroll
                    for (int s = 0; s < NS; s++)
#pragma unroll
                        for (int i = 0; i < VEC; i++)
                            if (ok[u]) acc[s][i] = fmaf(wv[u], v[u][s][i], acc[s][i]);
            }
        }
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = c0 + (lane + 32 * s) * VEC;
            if (col < a.d) {
                if (a.pre) {
#pragma unroll
                    for (int i = 0; i < VEC; i++) {
                        const int64_t off = n * a.d + col + i;
                        const float p = a.pre_dtype == SMLM_F32
                                            ? __ldg(static_cast<const float*>(a.pre) + off)
                                            : bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(a.pre) + off));
                        acc[s][i] = acc[s][i] * silu_bf16(p);
                    }
                }
                store_out<VEC>(a.out, a.out_dtype, n * a.d + col, acc[s]);
            }
        }
    }
}

template <typename TT, int VEC>
static int launch_bag_vec(BagArgs a, cudaStream_t st) {
    const int slots = (a.d + VEC - 1) / VEC;
    const int ns = (slots + 31) / 32;
    int blocks_needed;
    auto go = [&](auto NSc) {
        constexpr int NS = decltype(NSc)::value;
        a.col_block = 32 * VEC * NS;
        const int64_t tasks = a.n * ((a.d + a.col_block - 1) / a.col_block);
        const int64_t want = (tasks + 7) / 8;
        blocks_needed = (int)std::min<int64_t>(want, (int64_t)sm_count() * 16);
        if (blocks_needed < 1) blocks_needed = 1;
        bag_gather_kernel<TT, VEC, NS><<<blocks_needed, 256, 0, st>>>(a);
    };
    if (ns <= 1) go(std::integral_constant<int, 1>{});
    else if (ns == 2) go(std::integral_constant<int, 2>{});
    else if (ns == 3) go(std::integral_constant<int, 3>{});
    else go(std::integral_constant<int, 4>{});
    SMLM_LAUNCHED("bag_gather_kernel");
    return SMLM_OK;
}

// Few tokens (decoding, short prompts): one warp per (token, 512-byte column block). A warp-per-token gather
// keeps only a few rows in flight, so a token's lookups would cost one memory round trip per few rows. Here
// every valid lookup's slice of the column block is copied into shared memory with cp.async (16 bytes per lane,
// L2-only), up to SMALL_STAGES chunks of 32 lookups in flight at once, and then summed in lookup order: the same
// sequential fmaf chain per column as bag_gather_kernel, so the same bits. A lane reads back only the bytes it
// copied itself; the chunk's weights and valid marks go through shared memory to the whole warp.
constexpr int SMALL_STAGES = 4;
constexpr int SMALL_ROW_BYTES = 512;  // 32 lanes x 16 bytes

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait(int pending) {  // wait until at most `pending` groups are in flight
    if (pending <= 0) asm volatile("cp.async.wait_group 0;" ::: "memory");
    else if (pending == 1) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else if (pending == 2) asm volatile("cp.async.wait_group 2;" ::: "memory");
    else asm volatile("cp.async.wait_group 3;" ::: "memory");
}

template <typename TT>
__global__ void __launch_bounds__(32) bag_small_kernel(BagArgs a, int stages) {
    constexpr int VEC = 16 / sizeof(TT);
    extern __shared__ __align__(16) uint8_t small_buf[];                      // [stages][32][512]
    float* sw = reinterpret_cast<float*>(small_buf + stages * 32 * SMALL_ROW_BYTES);  // [stages][32] weights
    uint32_t* svalid = reinterpret_cast<uint32_t*>(sw + stages * 32);                 // [stages] valid lookups
    const int lane = threadIdx.x;
    const int nblk = (a.d + 32 * VEC - 1) / (32 * VEC);
    const int64_t n = blockIdx.x / nblk;
    const int col = (int)(blockIdx.x % nblk) * 32 * VEC + lane * VEC;
    const bool on = col < a.d;
    const TT* table = static_cast<const TT*>(a.table);
    const int nchunks = (a.k + 31) / 32;

    auto issue = [&](int ch) {
        const int slot = ch % stages;
        const int j = ch * 32 + lane;
        int64_t r = -1;
        float w = 0.f;
        if (j < a.k) {
            r = load_index(a.idx, a.idx32, n * a.k + j) - a.row_base;
            w = load_weight(a.w, a.w_dtype, n * a.k + j);
            if (r < 0 || r >= a.rows) {
                if (!a.skip_foreign) flag(a.status, SMLM_FLAG_INDEX_RANGE);
                r = -1;
            }
        }
        sw[slot * 32 + lane] = w;
        const uint32_t valid = __ballot_sync(FULL, r >= 0);
        if (lane == 0) svalid[slot] = valid;
        const int cnt = min(32, a.k - ch * 32);
        uint8_t* dst = small_buf + (size_t)slot * 32 * SMALL_ROW_BYTES + lane * 16;
        for (int u = 0; u < cnt; u++) {
            const int64_t ru = __shfl_sync(FULL, r, u);
            if (ru >= 0 && on) cp_async16(dst + u * SMALL_ROW_BYTES, table + ru * a.d + col);
        }
        cp_async_commit();
    };

    float acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; i++) acc[i] = 0.f;
    int issued = 0;
    for (; issued < min(stages, nchunks); issued++) issue(issued);
    for (int ch = 0; ch < nchunks; ch++) {
        cp_async_wait(issued - ch - 1);
        __syncwarp();
        const int slot = ch % stages;
        const int cnt = min(32, a.k - ch * 32);
        const uint8_t* src = small_buf + (size_t)slot * 32 * SMALL_ROW_BYTES + lane * 16;
        const uint32_t valid = svalid[slot];
        for (int u = 0; u < cnt; u++) {
            if (!((valid >> u) & 1u) || !on) continue;  // warp-uniform except for `on`
            const float w = sw[slot * 32 + u];
            float v[VEC];
            if constexpr (sizeof(TT) == 4) {
                const float4 x = *reinterpret_cast<const float4*>(src + u * SMALL_ROW_BYTES);
                v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
            } else {
                const uint4 x = *reinterpret_cast<const uint4*>(src + u * SMALL_ROW_BYTES);
                const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    v[2 * i] = bf16_bits_to_f32(xs[i] & 0xffffu);
                    v[2 * i + 1] = bf16_bits_to_f32(xs[i] >> 16);
                }
            }
#pragma unroll
            for (int i = 0; i < VEC; i++) acc[i] = fmaf(w, v[i], acc[i]);
        }
        __syncwarp();  // the slot is free again
        if (issued < nchunks) issue(issued++);
    }
    if (!on) return;
    if (a.pre) {
#pragma unroll
        for (int i = 0; i < VEC; i++) {
            const int64_t off = n * a.d + col + i;
            const float p = a.pre_dtype == SMLM_F32 ? __ldg(static_cast<const float*>(a.pre) + off)
                                                    : bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(a.pre) + off));
            acc[i] = acc[i] * silu_bf16(p);
        }
    }
    store_out<VEC>(a.out, a.out_dtype, n * a.d + col, acc);
}

// Token counts up to this take bag_small_kernel.
constexpr int64_t BAG_SMALL_N = 256;

template <typename TT>
static int launch_bag_small(BagArgs a, cudaStream_t st) {
    constexpr int VEC = 16 / sizeof(TT);
    const int stages = (int)std::min<int64_t>(SMALL_STAGES, (a.k + 31) / 32);
    const size_t smem = (size_t)stages * (32 * (SMALL_ROW_BYTES + 4) + 4);
    if (smem > 48 * 1024) {
        SMLM_CUDA(cudaFuncSetAttribute(bag_small_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    }
    const int64_t blocks = a.n * ((a.d + 32 * VEC - 1) / (32 * VEC));
    bag_small_kernel<TT><<<(unsigned)blocks, 32, smem, st>>>(a, stages);
    SMLM_LAUNCHED("bag_small_kernel");
    return SMLM_OK;
}

static int launch_bag(BagArgs a, int table_dtype, cudaStream_t st) {
    if (a.n == 0 || a.d == 0) return SMLM_OK;
    const uintptr_t tp = reinterpret_cast<uintptr_t>(a.table);
    const uintptr_t op = reinterpret_cast<uintptr_t>(a.out);
    if (a.n <= BAG_SMALL_N && a.k > 0 && tp % 16 == 0 && (a.out_dtype != SMLM_F32 || op % 16 == 0) &&
        (a.pre == nullptr || a.pre_dtype == SMLM_F32 || a.pre_dtype == SMLM_BF16)) {
        if (table_dtype == SMLM_F32 && a.d % 4 == 0) return launch_bag_small<float>(a, st);
        if (table_dtype == SMLM_BF16 && a.d % 8 == 0) return launch_bag_small<__nv_bfloat16>(a, st);
    }
    const bool out_vec_ok = a.out_dtype != SMLM_F32 || (op % 16 == 0);
    if (table_dtype == SMLM_F32) {
        if (a.d % 4 == 0 && tp % 16 == 0 && out_vec_ok) return launch_bag_vec<float, 4>(a, st);
        return launch_bag_vec<float, 1>(a, st);
    }
    if (a.d % 4 == 0 && tp % 8 == 0 && out_vec_ok) return launch_bag_vec<__nv_bfloat16, 4>(a, st);
    return launch_bag_vec<__nv_bfloat16, 1>(a, st);
}

// ------------------------------------------------------------------------------------------------------ q4
// Row r: d/2 bytes, byte i = (code of column i) | (code of column i + d/2) << 4, code = c + 8, value = c * s_r.
struct Q4Args {
    const int64_t* idx;
    const void* w;
    int w_dtype;
    const uint8_t* table;
    const uint16_t* scales;  // fp16 bits
    const void* pre;
    int pre_dtype;
    void* out;
    int out_dtype;
    int64_t n, rows;
    int k, d;
    int* status;
};

// One warp per token; lane s handles bytes [8 s, 8 s + 8) of the row (columns 8s.. and d/2 + 8s..), so one
// 8-byte load per lane per row; tokens with d/2 > 256 loop over byte blocks.
template <int VEC>
__global__ void __launch_bounds__(256) bag_q4_kernel(Q4Args a) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int dh = a.d / 2;
    const int blk = 32 * VEC;
    const int nblk = (dh + blk - 1) / blk;
    for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < a.n * nblk;
         task += warps) {
        const int64_t n = task / nblk;
        const int b0 = (int)(task % nblk) * blk + lane * VEC;
        float lo[VEC], hi[VEC];
#pragma unroll
        for (int i = 0; i < VEC; i++) lo[i] = hi[i] = 0.f;
        for (int j0 = 0; j0 < a.k; j0 += 32) {
            const int cnt = min(32, a.k - j0);
            int64_t my_r = -1;
            float my_w = 0.f;
            if (lane < cnt) {
                my_r = __ldg(a.idx + n * a.k + j0 + lane);
                my_w = load_weight(a.w, a.w_dtype, n * a.k + j0 + lane);
                if (my_r < 0 || my_r >= a.rows) {
                    flag(a.status, SMLM_FLAG_INDEX_RANGE);
                    my_r = -1;
                } else {
                    my_w = my_w * __half2float(__ushort_as_half(__ldg(a.scales + my_r)));
                }
            }
            for (int jj = 0; jj < cnt; jj++) {
                const int64_t r = __shfl_sync(FULL, my_r, jj);
                const float ws = __shfl_sync(FULL, my_w, jj);
                if (r < 0 || b0 >= dh) continue;
                uint8_t bytes[VEC];
                if constexpr (VEC == 8) {
                    uint2 x = __ldg(reinterpret_cast<const uint2*>(a.table + r * dh + b0));
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        bytes[i] = (x.x >> (8 * i)) & 0xff;
                        bytes[4 + i] = (x.y >> (8 * i)) & 0xff;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < VEC; i++) bytes[i] = b0 + i < dh ? __ldg(a.table + r * dh + b0 + i) : 8;
                }
#pragma unroll
                for (int i = 0; i < VEC; i++) {
                    lo[i] = fmaf(ws, (float)((int)(bytes[i] & 15) - 8), lo[i]);
                    hi[i] = fmaf(ws, (float)((int)(bytes[i] >> 4) - 8), hi[i]);
                }
            }
        }
#pragma unroll
        for (int half = 0; half < 2; half++) {
#pragma unroll
            for (int i = 0; i < VEC; i++) {
                if (b0 + i >= dh) continue;
                const int col = b0 + i + half * dh;
                float v = half ? hi[i] : lo[i];
                const int64_t off = n * a.d + col;
                if (a.pre) {
                    const float p = a.pre_dtype == SMLM_F32
                                        ? __ldg(static_cast<const float*>(a.pre) + off)
                                        : bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(a.pre) + off));
                    v = v * silu_bf16(p);
                }
                if (a.out_dtype == SMLM_F32) static_cast<float*>(a.out)[off] = v;
                else static_cast<uint16_t*>(a.out)[off] = (uint16_t)f32_to_bf16_bits(v);
            }
        }
    }
}

// One warp per row: scale from the element of largest |w| (first such column), then codes.
__global__ void __launch_bounds__(256) quantize_q4_kernel(const float* table, int64_t rows, int d,
                                                          uint8_t* packed, uint16_t* scales) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int dh = d / 2;
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float* row = table + r * d;
        float best = -1.f;
        int best_col = 0x7fffffff;
        for (int c = lane; c < d; c += 32) {
            const float a = fabsf(row[c]);
            if (a > best) { best = a; best_col = c; }  // first column of this lane's largest |w|
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(FULL, best, o);
            const int oc = __shfl_xor_sync(FULL, best_col, o);
            if (ob > best || (ob == best && oc < best_col)) { best = ob; best_col = oc; }
        }
        if (best_col >= d) best_col = 0;  // all-NaN row
        const float m = row[best_col];
        __half dh16 = __float2half_rn(m / -8.0f);
        if (__half2float(dh16) == 0.f) dh16 = __float2half_rn(1.0f);
        const float s = __half2float(dh16);
        for (int c = lane; c < dh; c += 32) {
            const float q0 = fminf(fmaxf(rintf(row[c] / s), -8.f), 7.f) + 8.f;
            const float q1 = fminf(fmaxf(rintf(row[c + dh] / s), -8.f), 7.f) + 8.f;
            packed[r * dh + c] = (uint8_t)((int)q0 | ((int)q1 << 4));
        }
        if (lane == 0) scales[r] = __half_as_ushort(dh16);
    }
}

// ---------------------------------------------------------------------------------------------- backward
constexpr uint32_t NO_ROW = 0xffffffffu;
constexpr int FLAG_TAIL = 1;  // chunk's last run continues into the next chunk; partial in carry_tail
constexpr int FLAG_MID = 2;   // the whole chunk is one run that started before and continues after

static int chunk_positions(int64_t m) { return m >= (1 << 20) ? 256 : 64; }

static int bit_width_u32(uint64_t x) {
    int b = 0;
    while (x) { b++; x >>= 1; }
    return b;
}

// skip_foreign: rows outside [row_base, row_base + rows) belong to other shards (past-the-end key, not flagged).
__global__ void bb_keys_kernel(const void* idx, int idx32, int64_t row_base, int skip_foreign, int64_t m,
                               int64_t rows, uint32_t* keys, uint32_t* pos, int* status) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < m; p += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = load_index(idx, idx32, p) - row_base;
        uint32_t key = (uint32_t)r;
        if (r < 0 || r >= rows) {
            if (!skip_foreign) flag(status, SMLM_FLAG_INDEX_RANGE);
            key = (uint32_t)rows;  // sorts after every valid row; skipped by the segment pass
        }
        keys[p] = key;
        pos[p] = (uint32_t)p;
    }
}

struct SegArgs {
    const uint32_t* keys;  // sorted rows
    const uint32_t* pos;   // positions (n * k + j), ascending within a row
    const void* g;         // grad_out (n, d), fp32 or bf16
    int g_dtype;
    const void* w;
    int w_dtype;
    const void* table;
    float* acc;
    uint8_t* touched;
    float* gw;
    float* carry_head;  // (chunks, d)
    float* carry_tail;  // (chunks, d)
    int* chunk_flags;   // (chunks,)
    float* sqnorm;      // optional (rows,): squared L2 norm of every accumulator row this call writes
    int first_writes;   // rows whose touched byte is 0 are written (not accumulated): they count as zero
    int64_t m, rows;
    int k, d, P;
    int64_t chunks;
    int all_fresh;      // every row counts as untouched (materialising a deferred backward)
};

// The fused optimizer pass over deferred row sums: each completed row sum goes straight into lazy Adam.
struct RowAdam {
    float *p, *m, *v;
    const float* scale_dev;
    float scale;
    AdamScalars s;
    void* copy;
    int copy_dtype;
    // the fused row-wise step (ROWS_ROWWISE): per-row state, kind and scalars (p, scale_dev and scale above)
    float* row_v;
    int32_t* row_count;
    int rw_kind;
    float rw_b2, rw_eps, rw_lr;
    // lazy Adam's six scalars in device memory instead of `s` (one_minus_b1, b2, one_minus_b2, bc2_sqrt, eps,
    // neg_step): a step replayed from a CUDA graph reads that step's values, written before the replay
    const float* s_dev;
};

__device__ __forceinline__ AdamScalars adam_scalars(const RowAdam& ad) {
    if (ad.s_dev == nullptr) return ad.s;
    return AdamScalars{ad.s_dev[0], ad.s_dev[1], ad.s_dev[2], ad.s_dev[3], ad.s_dev[4], ad.s_dev[5]};
}

// What the row-sum pass does with a completed row sum x (= 0 + the run's sum for a first touch):
constexpr int ROWS_WRITE = 0;  // acc[row] = x (or acc[row] + x), its squared norm, touched = 1
constexpr int ROWS_NORM = 1;   // only its squared norm and touched = 1 (deferred backward: acc stays untouched)
constexpr int ROWS_ADAM = 2;   // lazy Adam of the table row with gradient x, touched = 0
constexpr int ROWS_ROWWISE = 3;  // the row-wise (rowrms / rowadagrad) step of the table row with gradient x

// Parameters and moments of a touched row: read once and written once per step (streaming, evict-first).
__device__ __forceinline__ void ld_stream4(const float* p, float (&v)[4]) {
    const float4 x = __ldcs(reinterpret_cast<const float4*>(p));
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}

// One warp per chunk of P sorted positions. Each run of equal rows is summed in position order; runs that
// lie inside the chunk go straight into acc (they belong to this chunk alone: no atomics), the run that
// enters from the previous chunk goes to carry_head, the run that leaves to carry_tail (see fixup).
// Memory-level parallelism: a batch of 32 positions is loaded one per lane together with its weight and (first-
// touch mode) its row's touched byte; the next position's grad_out row and, when it starts a run, its table row
// are loaded while the current position is summed.
template <typename TT, typename GT, bool GW, int VEC, int NS>
__global__ void __launch_bounds__(128) bb_segment_kernel(SegArgs a) {
    const int lane = lane_id();
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= a.chunks) return;
    const TT* table = static_cast<const TT*>(a.table);
    const GT* g = static_cast<const GT*>(a.g);
    const int64_t start = c * a.P;
    const int64_t end = min(start + (int64_t)a.P, a.m);
    const uint32_t valid_lim = (uint32_t)a.rows;
    const uint32_t first_row = a.keys[start];
    if (first_row >= valid_lim && !GW) {  // only past-the-end keys from here on: nothing to add
        if (lane == 0) a.chunk_flags[c] = 0;
        return;
    }
    const uint32_t last_row = a.keys[end - 1];
    const uint32_t prev_row = start > 0 ? a.keys[start - 1] : NO_ROW;
    const uint32_t next_row = end < a.m ? a.keys[end] : NO_ROW;
    const bool head_cross = first_row < valid_lim && prev_row == first_row;
    const bool tail_cross = last_row < valid_lim && next_row == last_row;
    const bool mid = head_cross && tail_cross && first_row == last_row;
    int cflags = 0;

    uint32_t cur = NO_ROW;
    bool cur_fresh = false;  // first-touch mode: the current row had not been touched before this call
    float sum[NS][VEC], trow[NS][VEC];
#pragma unroll
    for (int s = 0; s < NS; s++)
#pragma unroll
        for (int i = 0; i < VEC; i++) sum[s][i] = trow[s][i] = 0.f;

    auto flush = [&]() {
        if (cur == NO_ROW || a.acc == nullptr) return;  // acc == NULL: per-sample-weight gradient only
        float* dst = nullptr;
        bool direct = false;
        float sq = 0.f;
        if (mid) {
            dst = a.carry_head + c * a.d;
            cflags |= FLAG_MID;
        } else if (head_cross && cur == first_row) {
            dst = a.carry_head + c * a.d;
        } else if (tail_cross && cur == last_row) {
            dst = a.carry_tail + c * a.d;
            cflags |= FLAG_TAIL;
        } else {
            dst = a.acc + (int64_t)cur * a.d;
            direct = true;
        }
        // a row seen for the first time since the optimizer step is written, not read (first_writes mode)
        const bool accumulate = direct && !cur_fresh;
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * VEC;
            if (col < a.d) {
                if constexpr (VEC == 4) {
                    float4* q = reinterpret_cast<float4*>(dst + col);
                    float4 x = accumulate ? *q : make_float4(0.f, 0.f, 0.f, 0.f);
                    x.x = x.x + sum[s][0]; x.y = x.y + sum[s][1]; x.z = x.z + sum[s][2]; x.w = x.w + sum[s][3];
                    *q = x;
                    sq = fmaf(x.x, x.x, sq); sq = fmaf(x.y, x.y, sq); sq = fmaf(x.z, x.z, sq); sq = fmaf(x.w, x.w, sq);
                } else {
#pragma unroll
                    for (int i = 0; i < VEC; i++) {
                        const float x = (accumulate ? dst[col + i] : 0.f) + sum[s][i];
                        dst[col + i] = x;
                        sq = fmaf(x, x, sq);
                    }
                }
            }
        }
        if (direct) {
            if (a.sqnorm) {
                sq = warp_sum(sq);
                if (lane == 0) a.sqnorm[cur] = sq;
            }
            if (lane == 0 && a.touched) a.touched[cur] = 1;
        }
    };
    auto load_g = [&](uint32_t p, float (&v)[NS][VEC]) {
        const int64_t tok = p / a.k;
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * VEC;
            if (col < a.d) Elt<GT>::template load<VEC>(g + tok * a.d + col, v[s]);
        }
    };
    auto load_t = [&](uint32_t row, float (&v)[NS][VEC]) {
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * VEC;
            if (col < a.d) Elt<TT>::template load<VEC>(table + (int64_t)row * a.d + col, v[s]);
        }
    };

    for (int64_t b = start; b < end; b += 32) {
        const int cnt = (int)min((int64_t)32, end - b);
        uint32_t my_key = NO_ROW, my_pos = 0;
        float my_w = 0.f;
        bool my_fresh = false;
        if (lane < cnt) {
            my_key = a.keys[b + lane];
            my_pos = a.pos[b + lane];
            if (my_key < valid_lim) {
                my_w = load_weight(a.w, a.w_dtype, my_pos);
                my_fresh = a.first_writes && a.touched && a.touched[my_key] == 0;
            }
        }
        float gn[NS][VEC], tn[NS][VEC];
        uint32_t row_n = __shfl_sync(FULL, my_key, 0);
        if (row_n < valid_lim) {
            load_g(__shfl_sync(FULL, my_pos, 0), gn);
            if (GW && row_n != cur) load_t(row_n, tn);
        }
        for (int t = 0; t < cnt; t++) {
            const uint32_t row = row_n;
            const uint32_t p = __shfl_sync(FULL, my_pos, t);
            const float wv = __shfl_sync(FULL, my_w, t);
            const bool fresh = __shfl_sync(FULL, (int)my_fresh, t) != 0;
            const bool live = row < valid_lim;  // else an out-of-range or skipped lookup (flagged at key build)
            if (live && row != cur) {
                flush();
                cur = row;
                cur_fresh = fresh;
#pragma unroll
                for (int s = 0; s < NS; s++)
#pragma unroll
                    for (int i = 0; i < VEC; i++) {
                        sum[s][i] = 0.f;
                        if (GW) trow[s][i] = tn[s][i];
                    }
            }
            float gv[NS][VEC];
#pragma unroll
            for (int s = 0; s < NS; s++)
#pragma unroll
                for (int i = 0; i < VEC; i++) gv[s][i] = gn[s][i];
            // issue the next position's loads before this position's arithmetic
            row_n = t + 1 < cnt ? __shfl_sync(FULL, my_key, t + 1) : NO_ROW;
            if (row_n < valid_lim) {
                load_g(__shfl_sync(FULL, my_pos, t + 1), gn);
                if (GW && row_n != row) load_t(row_n, tn);
            }
            if (!live) {
                if (GW && lane == 0) a.gw[p] = 0.f;
                continue;
            }
            float dot = 0.f;
#pragma unroll
            for (int s = 0; s < NS; s++) {
                const int col = (lane + 32 * s) * VEC;
                if (col < a.d) {
#pragma unroll
                    for (int i = 0; i < VEC; i++) {
                        sum[s][i] = fmaf(wv, gv[s][i], sum[s][i]);
                        if (GW) dot = fmaf(gv[s][i], trow[s][i], dot);
                    }
                }
            }
            if (GW) {
                dot = warp_sum(dot);
                if (lane == 0) a.gw[p] = dot;
            }
        }
    }
    flush();
    if (lane == 0) a.chunk_flags[c] = cflags;
}

// Per-sample-weight gradient, gather-shaped: gw[n, j] = <grad_out[n], table[row(n, j)]>. One warp per token
// holds the token's grad_out row in registers and walks its lookups in chunks of 32, four table rows in flight
// and their four dot products reduced together; lane j keeps the dot of lookup j, stored coalesced per chunk.
// Lookups outside the table (or outside the shard) get 0.
struct GwArgs {
    const void* g;
    const void* idx;
    int idx32;
    int64_t row_base;
    const void* table;
    float* gw;
    int64_t n, rows;
    int k, d;
};

template <typename TT, typename GT, int NS>
__global__ void __launch_bounds__(128) bb_gw_kernel(GwArgs a) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const TT* table = static_cast<const TT*>(a.table);
    const GT* g = static_cast<const GT*>(a.g);
    for (int64_t n = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < a.n; n += warps) {
        float gv[NS][4];
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * 4;
            if (col < a.d) Elt<GT>::template load<4>(g + n * a.d + col, gv[s]);
            else gv[s][0] = gv[s][1] = gv[s][2] = gv[s][3] = 0.f;
        }
        for (int j0 = 0; j0 < a.k; j0 += 32) {
            const int cnt = min(32, a.k - j0);
            int64_t my_r = -1;
            if (lane < cnt) {
                const int64_t r = load_index(a.idx, a.idx32, n * a.k + j0 + lane) - a.row_base;
                my_r = (r >= 0 && r < a.rows) ? r : -1;
            }
            float mine = 0.f;  // lane j: the dot of lookup j0 + j
#pragma unroll 1
            for (int jj = 0; jj < cnt; jj += 4) {
                float v[4][NS][4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int64_t r = __shfl_sync(FULL, my_r, (jj + u) & 31);  // -1 past cnt (lanes >= cnt)
#pragma unroll
                    for (int s = 0; s < NS; s++) {
                        const int col = (lane + 32 * s) * 4;
                        if (r >= 0 && col < a.d) Elt<TT>::template load<4>(table + r * a.d + col, v[u][s]);
                        else v[u][s][0] = v[u][s][1] = v[u][s][2] = v[u][s][3] = 0.f;
                    }
                }
                float dot[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    dot[u] = 0.f;
#pragma unroll
                    for (int s = 0; s < NS; s++)
#pragma unroll
                        for (int i = 0; i < 4; i++) dot[u] = fmaf(gv[s][i], v[u][s][i], dot[u]);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int u = 0; u < 4; u++) dot[u] += __shfl_xor_sync(FULL, dot[u], o);
#pragma unroll
                for (int u = 0; u < 4; u++)
                    if (lane == jj + u) mine = dot[u];
            }
            if (lane < cnt) a.gw[n * a.k + j0 + lane] = mine;
        }
    }
}

template <typename TT, typename GT>
static void launch_gw(GwArgs a, cudaStream_t st) {
    const int ns = (a.d + 127) / 128;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((a.n + 3) / 4, (int64_t)sm_count() * 32));
    if (ns <= 1) bb_gw_kernel<TT, GT, 1><<<blocks, 128, 0, st>>>(a);
    else if (ns == 2) bb_gw_kernel<TT, GT, 2><<<blocks, 128, 0, st>>>(a);
    else if (ns == 3) bb_gw_kernel<TT, GT, 3><<<blocks, 128, 0, st>>>(a);
    else bb_gw_kernel<TT, GT, 4><<<blocks, 128, 0, st>>>(a);
}

// The segment pass without the weight gradient (bb_gw_kernel computes it), with the per-position work cut down:
// per batch of 32 sorted positions each lane fetches one position's row, token (one division per lane),
// weight and first-touch flag; the warp then walks the batch's in-range prefix (out-of-range keys sort last)
// with the next position's grad_out row in flight in a second register buffer, adds w * grad_out row to the
// run's sum, and writes each finished run's row once (with its squared norm and touched flag). Same summation
// order and results as bb_segment_kernel.
template <typename GT, int NS, int MODE>
__global__ void __launch_bounds__(128) bb_rowsum_kernel(SegArgs a, RowAdam ad) {
    const int lane = lane_id();
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= a.chunks) return;
    const GT* g = static_cast<const GT*>(a.g);
    const int64_t start = c * a.P;
    const int64_t end = min(start + (int64_t)a.P, a.m);
    const uint32_t valid_lim = (uint32_t)a.rows;
    const uint32_t first_row = a.keys[start];
    if (first_row >= valid_lim) {
        if (lane == 0) a.chunk_flags[c] = 0;
        return;
    }
    const uint32_t last_row = a.keys[end - 1];
    const uint32_t prev_row = start > 0 ? a.keys[start - 1] : NO_ROW;
    const uint32_t next_row = end < a.m ? a.keys[end] : NO_ROW;
    const bool head_cross = prev_row == first_row;
    const bool tail_cross = last_row < valid_lim && next_row == last_row;
    const bool mid = head_cross && tail_cross && first_row == last_row;
    int cflags = 0;
    constexpr uint32_t FRESH = 0x80000000u;
    constexpr bool STEP = MODE == ROWS_ADAM || MODE == ROWS_ROWWISE;  // an optimizer step on the table row
    const float scale = STEP ? (ad.scale_dev ? *ad.scale_dev : ad.scale) : 1.f;
    const AdamScalars asc = MODE == ROWS_ADAM ? adam_scalars(ad) : AdamScalars{};

    uint32_t cur = NO_ROW;
    bool cur_fresh = false;
    float sum[NS][4];
    float pr[STEP ? NS : 1][4], mr[MODE == ROWS_ADAM ? NS : 1][4], vr[MODE == ROWS_ADAM ? NS : 1][4];
#pragma unroll
    for (int s = 0; s < NS; s++) sum[s][0] = sum[s][1] = sum[s][2] = sum[s][3] = 0.f;

    auto is_direct = [&](uint32_t row) {
        return !mid && !(head_cross && row == first_row) && !(tail_cross && row == last_row);
    };
    auto flush = [&]() {
        if (cur == NO_ROW) return;
        float* dst = nullptr;
        const bool direct = is_direct(cur);
        if (mid) {
            dst = a.carry_head + c * a.d;
            cflags |= FLAG_MID;
        } else if (head_cross && cur == first_row) {
            dst = a.carry_head + c * a.d;
        } else if (tail_cross && cur == last_row) {
            dst = a.carry_tail + c * a.d;
            cflags |= FLAG_TAIL;
        } else if (MODE == ROWS_WRITE) {
            dst = a.acc + (int64_t)cur * a.d;
        }
        const bool accumulate = MODE == ROWS_WRITE && direct && !cur_fresh;
        if constexpr (MODE == ROWS_ROWWISE) {
            if (direct) {
                // the gradient x = 0 + the run's sum, scaled; q = mean of its squares in the rowwise kernel's
                // order (slot by slot, summed in double), then the row's state and the parameter update
                double q = 0.0;
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    if ((lane + 32 * s) * 4 < a.d) {
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            sum[s][i] = __fmul_rn(__fadd_rn(0.f, sum[s][i]), scale);
                            q = fma((double)sum[s][i], (double)sum[s][i], q);
                        }
                    }
                }
                q = warp_sum_d(q) / (double)a.d;
                const float step = rowwise_state_step(ad.rw_kind, ad.rw_b2, ad.rw_eps, ad.rw_lr, ad.row_v,
                                                      ad.row_count, cur, q, lane);
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const int col = (lane + 32 * s) * 4;
                    if (col < a.d) {
                        float4 pn;
                        pn.x = __fsub_rn(pr[s][0], __fmul_rn(step, sum[s][0]));
                        pn.y = __fsub_rn(pr[s][1], __fmul_rn(step, sum[s][1]));
                        pn.z = __fsub_rn(pr[s][2], __fmul_rn(step, sum[s][2]));
                        pn.w = __fsub_rn(pr[s][3], __fmul_rn(step, sum[s][3]));
                        __stcs(reinterpret_cast<float4*>(ad.p + (int64_t)cur * a.d + col), pn);
                    }
                }
                if (lane == 0 && a.touched) a.touched[cur] = 0;
                return;
            }
        }
        float sq = 0.f;
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * 4;
            if (col < a.d) {
                if (!direct) {  // a partial of a run that crosses chunks: the fix-up completes it
                    *reinterpret_cast<float4*>(dst + col) = make_float4(sum[s][0], sum[s][1], sum[s][2], sum[s][3]);
                    continue;
                }
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                if (accumulate) x = *reinterpret_cast<float4*>(dst + col);
                x.x = x.x + sum[s][0]; x.y = x.y + sum[s][1]; x.z = x.z + sum[s][2]; x.w = x.w + sum[s][3];
                if constexpr (MODE == ROWS_WRITE) {
                    __stcs(reinterpret_cast<float4*>(dst + col), x);  // not read again until the optimizer step
                } else if constexpr (MODE == ROWS_ADAM) {
                    const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                    for (int i = 0; i < 4; i++) adam_update(asc, scale, pr[s][i], mr[s][i], vr[s][i], xs[i]);
                    const int64_t o = (int64_t)cur * a.d + col;
                    __stcs(reinterpret_cast<float4*>(ad.p + o), make_float4(pr[s][0], pr[s][1], pr[s][2], pr[s][3]));
                    __stcs(reinterpret_cast<float4*>(ad.m + o), make_float4(mr[s][0], mr[s][1], mr[s][2], mr[s][3]));
                    __stcs(reinterpret_cast<float4*>(ad.v + o), make_float4(vr[s][0], vr[s][1], vr[s][2], vr[s][3]));
                    if (ad.copy) store_out<4>(ad.copy, ad.copy_dtype, o, pr[s]);
                }
                if constexpr (!STEP) {
                    sq = fmaf(x.x, x.x, sq); sq = fmaf(x.y, x.y, sq); sq = fmaf(x.z, x.z, sq); sq = fmaf(x.w, x.w, sq);
                }
            }
        }
        if (direct) {
            if (!STEP && a.sqnorm) {
                sq = warp_sum(sq);
                if (lane == 0) a.sqnorm[cur] = sq;
            }
            if (lane == 0 && a.touched) a.touched[cur] = STEP ? 0 : 1;
        }
    };
    auto load_g = [&](uint32_t tokf, float (&v)[NS][4]) {
        const GT* src = g + (size_t)(tokf & ~FRESH) * a.d;
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * 4;
            if (col < a.d) Elt<GT>::template load<4>(src + col, v[s]);
        }
    };
    auto step = [&](uint32_t row, uint32_t tokf, float wv, const float (&gv)[NS][4]) {
        if (row != cur) {
            flush();
            cur = row;
            cur_fresh = (tokf & FRESH) != 0;
#pragma unroll
            for (int s = 0; s < NS; s++) sum[s][0] = sum[s][1] = sum[s][2] = sum[s][3] = 0.f;
            if constexpr (STEP) {
                if (is_direct(row)) {  // the row's parameters (and moments), in flight while its run is summed
                    const int64_t base = (int64_t)row * a.d;
#pragma unroll
                    for (int s = 0; s < NS; s++) {
                        const int col = (lane + 32 * s) * 4;
                        if (col < a.d) {
                            ld_stream4(ad.p + base + col, pr[s]);
                            if constexpr (MODE == ROWS_ADAM) {
                                ld_stream4(ad.m + base + col, mr[s]);
                                ld_stream4(ad.v + base + col, vr[s]);
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int s = 0; s < NS; s++)
#pragma unroll
            for (int i = 0; i < 4; i++) sum[s][i] = fmaf(wv, gv[s][i], sum[s][i]);
    };

    for (int64_t b = start; b < end; b += 32) {
        const int cnt = (int)min((int64_t)32, end - b);
        uint32_t my_key = NO_ROW, my_tokf = 0;
        float my_w = 0.f;
        if (lane < cnt) {
            my_key = a.keys[b + lane];
            if (my_key < valid_lim) {
                const uint32_t p = a.pos[b + lane];
                const bool fresh = MODE == ROWS_WRITE &&
                                   (a.all_fresh || (a.first_writes && a.touched && a.touched[my_key] == 0));
                my_tokf = p / (uint32_t)a.k | (fresh ? FRESH : 0u);
                my_w = load_weight(a.w, a.w_dtype, p);
            }
        }
        const int nv = __popc(__ballot_sync(FULL, my_key < valid_lim));  // in-range keys: a prefix
        if (nv == 0) break;
        float ga[NS][4], gb[NS][4];
        load_g(__shfl_sync(FULL, my_tokf, 0), ga);
        int t = 0;
        for (; t + 1 < nv; t += 2) {
            load_g(__shfl_sync(FULL, my_tokf, t + 1), gb);
            step(__shfl_sync(FULL, my_key, t), __shfl_sync(FULL, my_tokf, t), __shfl_sync(FULL, my_w, t), ga);
            if (t + 2 < nv) load_g(__shfl_sync(FULL, my_tokf, t + 2), ga);
            step(__shfl_sync(FULL, my_key, t + 1), __shfl_sync(FULL, my_tokf, t + 1), __shfl_sync(FULL, my_w, t + 1),
                 gb);
        }
        if (t < nv)
            step(__shfl_sync(FULL, my_key, t), __shfl_sync(FULL, my_tokf, t), __shfl_sync(FULL, my_w, t), ga);
    }
    flush();
    if (lane == 0) a.chunk_flags[c] = cflags;
}

// The backward's norm pass (MODE ROWS_NORM: per touched row the squared norm of its sum and the touched mark, the
// sum itself not stored) with the rows that a single lookup reads taken 32 at a time. Most rows of a step are read
// once; walking them one position per warp iteration, as bb_rowsum_kernel walks runs, spent most of the pass on
// per-position control. Here each batch of 32 sorted positions first finds its singletons (key different from
// both neighbours in the whole sorted list, so never a row that crosses a chunk border): the warp reads their
// gradient rows one after the other, coalesced, AHEAD rows in flight, each lane keeping lane-partials of all 32
// (the fmaf chain over its columns, in bb_rowsum_kernel's order), and a transposing butterfly leaves singleton j's
// total on lane j, added in the same tree as warp_sum. The other positions go through bb_rowsum_kernel's run
// walk. The same norms, bit for bit, as summing every row first (bb_rowsum_kernel's write path).
template <typename GT, int NS, int AHEAD>
__global__ void __launch_bounds__(128) bb_rownorm_kernel(SegArgs a) {
    const int lane = lane_id();
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= a.chunks) return;
    const GT* g = static_cast<const GT*>(a.g);
    const int64_t start = c * a.P;
    const int64_t end = min(start + (int64_t)a.P, a.m);
    const uint32_t valid_lim = (uint32_t)a.rows;
    const uint32_t first_row = a.keys[start];
    if (first_row >= valid_lim) {
        if (lane == 0) a.chunk_flags[c] = 0;
        return;
    }
    const uint32_t last_row = a.keys[end - 1];
    const uint32_t prev_row = start > 0 ? a.keys[start - 1] : NO_ROW;
    const uint32_t next_row = end < a.m ? a.keys[end] : NO_ROW;
    const bool head_cross = prev_row == first_row;
    const bool tail_cross = last_row < valid_lim && next_row == last_row;
    const bool mid = head_cross && tail_cross && first_row == last_row;
    int cflags = 0;

    uint32_t cur = NO_ROW;
    float sum[NS][4];
#pragma unroll
    for (int s = 0; s < NS; s++) sum[s][0] = sum[s][1] = sum[s][2] = sum[s][3] = 0.f;

    auto flush = [&]() {
        if (cur == NO_ROW) return;
        float* dst = nullptr;
        bool direct = false;
        if (mid) {
            dst = a.carry_head + c * a.d;
            cflags |= FLAG_MID;
        } else if (head_cross && cur == first_row) {
            dst = a.carry_head + c * a.d;
        } else if (tail_cross && cur == last_row) {
            dst = a.carry_tail + c * a.d;
            cflags |= FLAG_TAIL;
        } else {
            direct = true;
        }
        float sq = 0.f;
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * 4;
            if (col < a.d) {
                if (!direct) {
                    *reinterpret_cast<float4*>(dst + col) = make_float4(sum[s][0], sum[s][1], sum[s][2], sum[s][3]);
                    continue;
                }
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                x.x = x.x + sum[s][0]; x.y = x.y + sum[s][1]; x.z = x.z + sum[s][2]; x.w = x.w + sum[s][3];
                sq = fmaf(x.x, x.x, sq); sq = fmaf(x.y, x.y, sq); sq = fmaf(x.z, x.z, sq); sq = fmaf(x.w, x.w, sq);
            }
        }
        if (direct) {
            if (a.sqnorm) {
                sq = warp_sum(sq);
                if (lane == 0) a.sqnorm[cur] = sq;
            }
            if (lane == 0 && a.touched) a.touched[cur] = 1;
        }
    };
    auto load_g = [&](uint32_t tok, float (&v)[NS][4]) {
        const GT* src = g + (size_t)tok * a.d;
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int col = (lane + 32 * s) * 4;
            if (col < a.d) Elt<GT>::template load<4>(src + col, v[s]);
        }
    };
    auto step = [&](uint32_t row, float wv, const float (&gv)[NS][4]) {
        if (row != cur) {
            flush();
            cur = row;
#pragma unroll
            for (int s = 0; s < NS; s++) sum[s][0] = sum[s][1] = sum[s][2] = sum[s][3] = 0.f;
        }
#pragma unroll
        for (int s = 0; s < NS; s++)
#pragma unroll
            for (int i = 0; i < 4; i++) sum[s][i] = fmaf(wv, gv[s][i], sum[s][i]);
    };

    for (int64_t b = start; b < end; b += 32) {
        const int cnt = (int)min((int64_t)32, end - b);
        uint32_t my_key = NO_ROW, my_tok = 0;
        float my_w = 0.f;
        if (lane < cnt) {
            my_key = a.keys[b + lane];
            if (my_key < valid_lim) {
                const uint32_t p = a.pos[b + lane];
                my_tok = p / (uint32_t)a.k;
                my_w = load_weight(a.w, a.w_dtype, p);
            }
        }
        const unsigned valid = __ballot_sync(FULL, my_key < valid_lim);  // in-range keys: a prefix
        if (valid == 0) break;
        // neighbours in the whole sorted list (across batch and chunk borders)
        uint32_t before = __shfl_up_sync(FULL, my_key, 1), after = __shfl_down_sync(FULL, my_key, 1);
        if (lane == 0) before = b > 0 ? a.keys[b - 1] : NO_ROW;
        if (lane == cnt - 1) after = b + cnt < a.m ? a.keys[b + cnt] : NO_ROW;
        const bool single = my_key < valid_lim && my_key != before && my_key != after;
        const unsigned smask = __ballot_sync(FULL, single);
        const unsigned wmask = valid & ~smask;  // positions for the run walk, in order
        if (smask) {
            // lane j takes the j-th singleton's row, token and weight
            const int src = __fns(smask, 0, lane + 1);
            const int ns1 = __popc(smask);
            const uint32_t srow = __shfl_sync(FULL, my_key, src & 31);
            const uint32_t stok = __shfl_sync(FULL, my_tok, src & 31);
            const float sw = __shfl_sync(FULL, my_w, src & 31);
            // gradient rows AHEAD singletons ahead, in a register ring (indices fixed at compile time)
            float part[32];
            float gbuf[AHEAD + 1][NS][4];
#pragma unroll
            for (int j = 0; j < AHEAD; j++)
                if (j < ns1) load_g(__shfl_sync(FULL, stok, j), gbuf[j]);
#pragma unroll
            for (int j = 0; j < 32; j++) {
                part[j] = 0.f;
                if (j < ns1) {  // warp-uniform
                    if (j + AHEAD < ns1) load_g(__shfl_sync(FULL, stok, j + AHEAD), gbuf[(j + AHEAD) % (AHEAD + 1)]);
                    const float wj = __shfl_sync(FULL, sw, j);
                    float sq = 0.f;
#pragma unroll
                    for (int s = 0; s < NS; s++) {
                        if ((lane + 32 * s) * 4 < a.d) {
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                const float x = fmaf(wj, gbuf[j % (AHEAD + 1)][s][i], 0.f);
                                sq = fmaf(x, x, sq);
                            }
                        }
                    }
                    part[j] = sq;
                }
            }
            // transposing butterfly: after the level with offset o, a lane holds the values of the singletons whose
            // bit log2(o) equals its own, each the sum of its own and its partner's; finally singleton `lane`
#pragma unroll
            for (int o = 16, n = 16; o > 0; o >>= 1, n >>= 1) {
                const bool upper = (lane & o) != 0;
#pragma unroll
                for (int j = 0; j < n; j++) {
                    const float send = upper ? part[j] : part[j + n];
                    const float keep = upper ? part[j + n] : part[j];
                    part[j] = keep + __shfl_xor_sync(FULL, send, o);
                }
            }
            if (lane < ns1) {
                if (a.sqnorm) a.sqnorm[srow] = part[0];
                if (a.touched) a.touched[srow] = 1;
            }
        }
        if (wmask == 0) continue;
        const int src = __fns(wmask, 0, lane + 1);
        const int nw = __popc(wmask);
        const uint32_t wkey = __shfl_sync(FULL, my_key, src & 31);
        const uint32_t wtok = __shfl_sync(FULL, my_tok, src & 31);
        const float wwt = __shfl_sync(FULL, my_w, src & 31);
        float ga[NS][4], gb[NS][4];
        load_g(__shfl_sync(FULL, wtok, 0), ga);
        int t = 0;
        for (; t + 1 < nw; t += 2) {
            load_g(__shfl_sync(FULL, wtok, t + 1), gb);
            step(__shfl_sync(FULL, wkey, t), __shfl_sync(FULL, wwt, t), ga);
            if (t + 2 < nw) load_g(__shfl_sync(FULL, wtok, t + 2), ga);
            step(__shfl_sync(FULL, wkey, t + 1), __shfl_sync(FULL, wwt, t + 1), gb);
        }
        if (t < nw) step(__shfl_sync(FULL, wkey, t), __shfl_sync(FULL, wwt, t), ga);
    }
    flush();
    if (lane == 0) a.chunk_flags[c] = cflags;
}

// bb_rowsum_kernel with four chunks per warp, one per quarter-warp (8 lanes x 4 NSQ columns hold a row): the
// quarters run the same instruction stream on different chunks, so the per-position control (shuffles, run
// tests, loop) serves four positions, and a warp keeps four rows in flight. Same summation order and results.
template <typename GT, int NSQ>
__global__ void __launch_bounds__(128) bb_rowsum4_kernel(SegArgs a) {
    const int lane = lane_id();
    const int ql = lane & 7;
    const int quarter = lane >> 3;
    const unsigned qmask = 0xffu << (8 * quarter);
    const int64_t c = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4 + quarter;
    if (c >= a.chunks) return;
    const GT* g = static_cast<const GT*>(a.g);
    const int64_t start = c * a.P;
    const int64_t end = min(start + (int64_t)a.P, a.m);
    const uint32_t valid_lim = (uint32_t)a.rows;
    const uint32_t first_row = a.keys[start];
    if (first_row >= valid_lim) {
        if (ql == 0) a.chunk_flags[c] = 0;
        return;
    }
    const uint32_t last_row = a.keys[end - 1];
    const uint32_t prev_row = start > 0 ? a.keys[start - 1] : NO_ROW;
    const uint32_t next_row = end < a.m ? a.keys[end] : NO_ROW;
    const bool head_cross = prev_row == first_row;
    const bool tail_cross = last_row < valid_lim && next_row == last_row;
    const bool mid = head_cross && tail_cross && first_row == last_row;
    int cflags = 0;
    constexpr uint32_t FRESH = 0x80000000u;

    uint32_t cur = NO_ROW;
    bool cur_fresh = false;
    float sum[NSQ][4];
#pragma unroll
    for (int s = 0; s < NSQ; s++) sum[s][0] = sum[s][1] = sum[s][2] = sum[s][3] = 0.f;

    auto flush = [&]() {
        if (cur == NO_ROW) return;
        float* dst;
        bool direct = false;
        if (mid) {
            dst = a.carry_head + c * a.d;
            cflags |= FLAG_MID;
        } else if (head_cross && cur == first_row) {
            dst = a.carry_head + c * a.d;
        } else if (tail_cross && cur == last_row) {
            dst = a.carry_tail + c * a.d;
            cflags |= FLAG_TAIL;
        } else {
            dst = a.acc + (int64_t)cur * a.d;
            direct = true;
        }
        const bool accumulate = direct && !cur_fresh;
        float sq = 0.f;
#pragma unroll
        for (int s = 0; s < NSQ; s++) {
            const int col = (ql + 8 * s) * 4;
            if (col < a.d) {
                float4* q = reinterpret_cast<float4*>(dst + col);
                float4 x = accumulate ? *q : make_float4(0.f, 0.f, 0.f, 0.f);
                x.x = x.x + sum[s][0]; x.y = x.y + sum[s][1]; x.z = x.z + sum[s][2]; x.w = x.w + sum[s][3];
                *q = x;
                sq = fmaf(x.x, x.x, sq); sq = fmaf(x.y, x.y, sq); sq = fmaf(x.z, x.z, sq); sq = fmaf(x.w, x.w, sq);
            }
        }
        if (direct) {
            if (a.sqnorm) {
#pragma unroll
                for (int o = 4; o > 0; o >>= 1) sq += __shfl_xor_sync(qmask, sq, o);
                if (ql == 0) a.sqnorm[cur] = sq;
            }
            if (ql == 0 && a.touched) a.touched[cur] = 1;
        }
    };

    for (int64_t b = start; b < end; b += 8) {
        const int cnt = (int)min((int64_t)8, end - b);
        uint32_t my_key = NO_ROW, my_tokf = 0;
        float my_w = 0.f;
        if (ql < cnt) {
            my_key = a.keys[b + ql];
            if (my_key < valid_lim) {
                const uint32_t p = a.pos[b + ql];
                const bool fresh = a.first_writes && a.touched && a.touched[my_key] == 0;
                my_tokf = p / (uint32_t)a.k | (fresh ? FRESH : 0u);
                my_w = load_weight(a.w, a.w_dtype, p);
            }
        }
        const int nv = __popc((__ballot_sync(qmask, my_key < valid_lim) >> (8 * quarter)) & 0xffu);
        if (nv == 0) break;
        for (int t = 0; t < nv; t++) {
            const uint32_t row = __shfl_sync(qmask, my_key, t, 8);
            const uint32_t tokf = __shfl_sync(qmask, my_tokf, t, 8);
            const float wv = __shfl_sync(qmask, my_w, t, 8);
            float gv[NSQ][4];
            const GT* src = g + (size_t)(tokf & ~FRESH) * a.d;
#pragma unroll
            for (int s = 0; s < NSQ; s++) {
                const int col = (ql + 8 * s) * 4;
                if (col < a.d) Elt<GT>::template load<4>(src + col, gv[s]);
                else gv[s][0] = gv[s][1] = gv[s][2] = gv[s][3] = 0.f;
            }
            if (row != cur) {
                flush();
                cur = row;
                cur_fresh = (tokf & FRESH) != 0;
#pragma unroll
                for (int s = 0; s < NSQ; s++) sum[s][0] = sum[s][1] = sum[s][2] = sum[s][3] = 0.f;
            }
#pragma unroll
            for (int s = 0; s < NSQ; s++)
#pragma unroll
                for (int i = 0; i < 4; i++) sum[s][i] = fmaf(wv, gv[s][i], sum[s][i]);
        }
    }
    flush();
    if (ql == 0) a.chunk_flags[c] = cflags;
}

// Completes the runs that cross chunk borders, in chunk order: tail of the run's first chunk, the full
// chunks it covers, then the head of the chunk where it ends; then does with the row what the row-sum pass does
// with a direct row (MODE).
template <int VEC, int MODE>
__global__ void __launch_bounds__(256) bb_fixup_kernel(SegArgs a, RowAdam ad) {
    const int lane = lane_id();
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= a.chunks || (MODE == ROWS_WRITE && a.acc == nullptr)) return;
    if (!(a.chunk_flags[c] & FLAG_TAIL)) return;
    const int64_t end = min((c + 1) * a.P, a.m);
    const uint32_t row = a.keys[end - 1];
    const bool accumulate = MODE == ROWS_WRITE && !a.all_fresh &&
                            !(a.first_writes && a.touched && a.touched[row] == 0);
    const float scale = (MODE == ROWS_ADAM || MODE == ROWS_ROWWISE) ? (ad.scale_dev ? *ad.scale_dev : ad.scale) : 1.f;
    const AdamScalars asc = MODE == ROWS_ADAM ? adam_scalars(ad) : AdamScalars{};
    // the row's total over its chunks, columns col0 .. col0 + VEC - 1, in chunk order
    auto total = [&](int col0, float (&tot)[VEC]) {
#pragma unroll
        for (int i = 0; i < VEC; i++) tot[i] = a.carry_tail[c * a.d + col0 + i];
        int64_t c2 = c + 1;
        while (c2 < a.chunks && (a.chunk_flags[c2] & FLAG_MID)) {
#pragma unroll
            for (int i = 0; i < VEC; i++) tot[i] = tot[i] + a.carry_head[c2 * a.d + col0 + i];
            c2++;
        }
        if (c2 < a.chunks) {
#pragma unroll
            for (int i = 0; i < VEC; i++) tot[i] = tot[i] + a.carry_head[c2 * a.d + col0 + i];
        }
    };
    if constexpr (MODE == ROWS_ROWWISE) {
        // two passes over the row: the mean square q first (rowwise kernel order), then the parameter update
        double q = 0.0;
        for (int col0 = lane * VEC; col0 < a.d; col0 += 32 * VEC) {
            float tot[VEC];
            total(col0, tot);
#pragma unroll
            for (int i = 0; i < VEC; i++) {
                const float gk = __fmul_rn(__fadd_rn(0.f, tot[i]), scale);
                q = fma((double)gk, (double)gk, q);
            }
        }
        q = warp_sum_d(q) / (double)a.d;
        const float step = rowwise_state_step(ad.rw_kind, ad.rw_b2, ad.rw_eps, ad.rw_lr, ad.row_v, ad.row_count,
                                              row, q, lane);
        for (int col0 = lane * VEC; col0 < a.d; col0 += 32 * VEC) {
            float tot[VEC];
            total(col0, tot);
            const int64_t o = (int64_t)row * a.d + col0;
#pragma unroll
            for (int i = 0; i < VEC; i++)
                ad.p[o + i] = __fsub_rn(ad.p[o + i], __fmul_rn(step, __fmul_rn(__fadd_rn(0.f, tot[i]), scale)));
        }
        if (lane == 0 && a.touched) a.touched[row] = 0;
        return;
    }
    float sq = 0.f;
    for (int col0 = lane * VEC; col0 < a.d; col0 += 32 * VEC) {
        float tot[VEC];
        total(col0, tot);
        const int64_t o = (int64_t)row * a.d + col0;
#pragma unroll
        for (int i = 0; i < VEC; i++) {
            const float x = (accumulate ? a.acc[o + i] : 0.f) + tot[i];
            if constexpr (MODE == ROWS_WRITE) a.acc[o + i] = x;
            if constexpr (MODE == ROWS_ADAM) {
                float p = ad.p[o + i], m = ad.m[o + i], v = ad.v[o + i];
                adam_update(asc, scale, p, m, v, x);
                ad.p[o + i] = p;
                ad.m[o + i] = m;
                ad.v[o + i] = v;
                if (ad.copy) {
                    if (ad.copy_dtype == SMLM_BF16) static_cast<uint16_t*>(ad.copy)[o + i] = (uint16_t)f32_to_bf16_bits(p);
                    else static_cast<float*>(ad.copy)[o + i] = p;
                }
            } else {
                sq = fmaf(x, x, sq);
            }
        }
    }
    if (MODE != ROWS_ADAM && a.sqnorm) {
        sq = warp_sum(sq);
        if (lane == 0) a.sqnorm[row] = sq;
    }
    if (lane == 0 && a.touched) a.touched[row] = MODE == ROWS_ADAM ? 0 : 1;
}

// The row-sum pass for a deferred backward (MODE ROWS_NORM) or the fused optimizer step (ROWS_ADAM): rows of
// 16-byte-aligned float4 groups only, at most 512 wide (the caller checks).
template <typename GT, int MODE>
static int launch_rows_mode(SegArgs a, RowAdam ad, cudaStream_t st) {
    const int ns = (a.d / 4 + 31) / 32;
    const int blocks = (int)((a.chunks + 3) / 4);
    if constexpr (MODE == ROWS_NORM) {
        if (ns <= 1) bb_rownorm_kernel<GT, 1, 2><<<blocks, 128, 0, st>>>(a);
        else if (ns == 2) bb_rownorm_kernel<GT, 2, 2><<<blocks, 128, 0, st>>>(a);
        else if (ns == 3) bb_rownorm_kernel<GT, 3, 2><<<blocks, 128, 0, st>>>(a);
        else bb_rownorm_kernel<GT, 4, 2><<<blocks, 128, 0, st>>>(a);
        SMLM_LAUNCHED("bb_rownorm_kernel");
    } else {
        if (ns <= 1) bb_rowsum_kernel<GT, 1, MODE><<<blocks, 128, 0, st>>>(a, ad);
        else if (ns == 2) bb_rowsum_kernel<GT, 2, MODE><<<blocks, 128, 0, st>>>(a, ad);
        else if (ns == 3) bb_rowsum_kernel<GT, 3, MODE><<<blocks, 128, 0, st>>>(a, ad);
        else bb_rowsum_kernel<GT, 4, MODE><<<blocks, 128, 0, st>>>(a, ad);
        SMLM_LAUNCHED("bb_rowsum_kernel");
    }
    bb_fixup_kernel<4, MODE><<<(int)((a.chunks + 7) / 8), 256, 0, st>>>(a, ad);
    SMLM_LAUNCHED("bb_fixup_kernel");
    return SMLM_OK;
}

static int invalid_width(int64_t d) {
    set_error("row-sparse backward: rows of %lld values are wider than the supported %d", (long long)d,
              SMLM_MAX_ROW_WIDTH);
    return SMLM_ERR_INVALID;
}

template <typename TT, typename GT, bool GW, int VEC>
static int launch_segment(SegArgs a, cudaStream_t st) {
    const int slots = (a.d + VEC - 1) / VEC;
    const int ns = (slots + 31) / 32;
    const int blocks = (int)((a.chunks + 3) / 4);
    const RowAdam none{};
    if (!GW && VEC == 4 && ns <= 1 && sizeof(GT) == 2 && a.acc != nullptr) {
        // short bf16 rows (the scoring backward's 128-wide key rows): four chunks per warp (measured faster);
        // wide fp32 rows keep one chunk per warp (measured faster there)
        bb_rowsum4_kernel<GT, 4><<<(int)((a.chunks + 15) / 16), 128, 0, st>>>(a);
        SMLM_LAUNCHED("bb_rowsum4_kernel");
    } else if (!GW && VEC == 4 && ns <= 4 && a.acc != nullptr) {
        if (ns <= 1) bb_rowsum_kernel<GT, 1, ROWS_WRITE><<<blocks, 128, 0, st>>>(a, none);
        else if (ns == 2) bb_rowsum_kernel<GT, 2, ROWS_WRITE><<<blocks, 128, 0, st>>>(a, none);
        else if (ns == 3) bb_rowsum_kernel<GT, 3, ROWS_WRITE><<<blocks, 128, 0, st>>>(a, none);
        else bb_rowsum_kernel<GT, 4, ROWS_WRITE><<<blocks, 128, 0, st>>>(a, none);
        SMLM_LAUNCHED("bb_rowsum_kernel");
    } else if (ns <= 1) bb_segment_kernel<TT, GT, GW, VEC, 1><<<blocks, 128, 0, st>>>(a);
    else if (ns == 2) bb_segment_kernel<TT, GT, GW, VEC, 2><<<blocks, 128, 0, st>>>(a);
    else if (ns == 3) bb_segment_kernel<TT, GT, GW, VEC, 3><<<blocks, 128, 0, st>>>(a);
    else if (ns == 4) bb_segment_kernel<TT, GT, GW, VEC, 4><<<blocks, 128, 0, st>>>(a);
    else {
        // scalar rows (widths that are not a multiple of 4, or unaligned data) up to SMLM_MAX_ROW_WIDTH
        if constexpr (VEC == 1) {
            if (ns <= 8) bb_segment_kernel<TT, GT, GW, 1, 8><<<blocks, 128, 0, st>>>(a);
            else if (ns <= 16) bb_segment_kernel<TT, GT, GW, 1, 16><<<blocks, 128, 0, st>>>(a);
            else return invalid_width(a.d);
        } else {
            return invalid_width(a.d);
        }
    }
    SMLM_LAUNCHED("bb_segment_kernel");
    bb_fixup_kernel<VEC, ROWS_WRITE><<<(int)((a.chunks + 7) / 8), 256, 0, st>>>(a, none);
    SMLM_LAUNCHED("bb_fixup_kernel");
    return SMLM_OK;
}

template <typename TT, int VEC>
static int launch_segment_g(SegArgs a, cudaStream_t st) {
    if (a.g_dtype == SMLM_F32)
        return a.gw ? launch_segment<TT, float, true, VEC>(a, st) : launch_segment<TT, float, false, VEC>(a, st);
    return a.gw ? launch_segment<TT, __nv_bfloat16, true, VEC>(a, st)
                : launch_segment<TT, __nv_bfloat16, false, VEC>(a, st);
}

struct BackwardPlan {
    int64_t m;
    int P;
    int64_t chunks;
    int end_bit;
    size_t sort_bytes;
};

static BackwardPlan plan_backward(int64_t n, int64_t k, int64_t rows) {
    BackwardPlan p;
    p.m = n * k;
    p.P = chunk_positions(p.m);
    p.chunks = (p.m + p.P - 1) / p.P;
    p.end_bit = bit_width_u32((uint64_t)rows);
    p.sort_bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, p.sort_bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                    (const uint32_t*)nullptr, (uint32_t*)nullptr, (int)std::max<int64_t>(p.m, 1),
                                    0, std::max(p.end_bit, 1));
    return p;
}

struct BackwardBufs {
    uint32_t *keys_in, *keys_out, *pos_in, *pos_out;
    void* sort_tmp;
    float *carry_head, *carry_tail;
    int* flags;
};

// Carves the workspace (base == nullptr: only computes the size, returned).
static size_t layout_backward(const BackwardPlan& p, int64_t d, void* base, BackwardBufs* b) {
    size_t off = 0;
    char* c = static_cast<char*>(base);
    auto take = [&](size_t bytes) -> void* {
        off = (off + 255) & ~size_t(255);
        void* ptr = c ? c + off : nullptr;
        off += bytes;
        return ptr;
    };
    b->keys_in = static_cast<uint32_t*>(take(sizeof(uint32_t) * p.m));
    b->keys_out = static_cast<uint32_t*>(take(sizeof(uint32_t) * p.m));
    b->pos_in = static_cast<uint32_t*>(take(sizeof(uint32_t) * p.m));
    b->pos_out = static_cast<uint32_t*>(take(sizeof(uint32_t) * p.m));
    b->sort_tmp = take(p.sort_bytes);
    b->carry_head = static_cast<float*>(take(sizeof(float) * p.chunks * d));
    b->carry_tail = static_cast<float*>(take(sizeof(float) * p.chunks * d));
    b->flags = static_cast<int*>(take(sizeof(int) * p.chunks));
    return off;
}

}  // namespace smlm

using namespace smlm;

extern "C" int smlm_bag_forward(const int64_t* indices, const void* weights, int weights_dtype, const void* table,
                                int table_dtype, int64_t n, int64_t k, int64_t rows, int64_t d, void* out,
                                int out_dtype, int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && k >= 0 && rows >= 0 && d >= 0, "bag_forward: negative size");
    SMLM_CHECK_ARG(table_dtype == SMLM_F32 || table_dtype == SMLM_BF16, "bag_forward: table must be fp32 or bf16");
    SMLM_CHECK_ARG(weights_dtype == SMLM_F32 || weights_dtype == SMLM_BF16, "bag_forward: weights must be fp32 or bf16");
    SMLM_CHECK_ARG(out_dtype == SMLM_F32 || out_dtype == SMLM_BF16, "bag_forward: out must be fp32 or bf16");
    SMLM_CHECK_ARG(d < (1 << 30) && k < (1 << 30), "bag_forward: d or k too large");
    if (n == 0 || d == 0) return SMLM_OK;
    SMLM_CHECK_ARG(indices && table && out && (k == 0 || weights), "bag_forward: null pointer");
    BagArgs a{indices, 0, 0, 0, weights, weights_dtype, table, nullptr, SMLM_F32, out, out_dtype, n, rows, (int)k,
              (int)d, 0, status};
    return launch_bag(a, table_dtype, as_stream(stream));
}

extern "C" int smlm_shard_bag_forward(const void* indices, int index_dtype, int64_t row_base, const void* weights,
                                      int weights_dtype, const void* table_shard, int table_dtype, int64_t n,
                                      int64_t k, int64_t shard_rows, int64_t d, void* out, int out_dtype,
                                      void* stream) {
    SMLM_CHECK_ARG(n >= 0 && k >= 0 && shard_rows >= 0 && d >= 0 && row_base >= 0, "shard_bag_forward: negative size");
    SMLM_CHECK_ARG(index_dtype == SMLM_I32 || index_dtype == SMLM_I64, "shard_bag_forward: int32 or int64 indices");
    SMLM_CHECK_ARG(table_dtype == SMLM_F32 || table_dtype == SMLM_BF16, "shard_bag_forward: table must be fp32 or bf16");
    SMLM_CHECK_ARG(weights_dtype == SMLM_F32 || weights_dtype == SMLM_BF16,
                   "shard_bag_forward: weights must be fp32 or bf16");
    SMLM_CHECK_ARG(out_dtype == SMLM_F32 || out_dtype == SMLM_BF16, "shard_bag_forward: out must be fp32 or bf16");
    SMLM_CHECK_ARG(d < (1 << 30) && k < (1 << 30), "shard_bag_forward: d or k too large");
    if (n == 0 || d == 0) return SMLM_OK;
    SMLM_CHECK_ARG(indices && out && (k == 0 || weights) && (table_shard || shard_rows == 0),
                   "shard_bag_forward: null pointer");
    BagArgs a{indices, index_dtype == SMLM_I32, row_base, 1, weights, weights_dtype, table_shard, nullptr, SMLM_F32,
              out, out_dtype, n, shard_rows, (int)k, (int)d, 0, nullptr};
    return launch_bag(a, table_dtype, as_stream(stream));
}

extern "C" int smlm_bag_infer(const int64_t* indices, const void* weights, int weights_dtype, const void* table,
                              int table_dtype, const void* scales, const void* pre, int pre_dtype, int64_t n,
                              int64_t k, int64_t rows, int64_t d, void* out, int out_dtype, int* status,
                              void* stream) {
    SMLM_CHECK_ARG(n >= 0 && k >= 0 && rows >= 0 && d >= 0, "bag_infer: negative size");
    SMLM_CHECK_ARG(table_dtype == SMLM_F32 || table_dtype == SMLM_BF16 || table_dtype == SMLM_Q4,
                   "bag_infer: table must be fp32, bf16 or q4");
    SMLM_CHECK_ARG(weights_dtype == SMLM_F32 || weights_dtype == SMLM_BF16, "bag_infer: weights must be fp32 or bf16");
    SMLM_CHECK_ARG(out_dtype == SMLM_F32 || out_dtype == SMLM_BF16, "bag_infer: out must be fp32 or bf16");
    SMLM_CHECK_ARG(pre == nullptr || pre_dtype == SMLM_F32 || pre_dtype == SMLM_BF16, "bag_infer: pre must be fp32 or bf16");
    SMLM_CHECK_ARG(table_dtype != SMLM_Q4 || (d % 2 == 0 && scales != nullptr), "bag_infer: q4 needs an even width and scales");
    SMLM_CHECK_ARG(d < (1 << 30) && k < (1 << 30), "bag_infer: d or k too large");
    if (n == 0 || d == 0) return SMLM_OK;
    SMLM_CHECK_ARG(indices && table && out && (k == 0 || weights), "bag_infer: null pointer");
    cudaStream_t st = as_stream(stream);
    if (table_dtype == SMLM_Q4) {
        Q4Args a{indices, weights, weights_dtype, static_cast<const uint8_t*>(table),
                 static_cast<const uint16_t*>(scales), pre, pre_dtype, out, out_dtype, n, rows, (int)k, (int)d,
                 status};
        const int dh = (int)(d / 2);
        const bool vec = dh % 8 == 0 && reinterpret_cast<uintptr_t>(table) % 8 == 0;
        const int blk = 32 * (vec ? 8 : 1);
        const int64_t tasks = n * ((dh + blk - 1) / blk);
        const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((tasks + 7) / 8, (int64_t)sm_count() * 16));
        if (vec) bag_q4_kernel<8><<<blocks, 256, 0, st>>>(a);
        else bag_q4_kernel<1><<<blocks, 256, 0, st>>>(a);
        SMLM_LAUNCHED("bag_q4_kernel");
        return SMLM_OK;
    }
    BagArgs a{indices, 0, 0, 0, weights, weights_dtype, table, pre, pre_dtype, out, out_dtype, n, rows, (int)k,
              (int)d, 0, status};
    return launch_bag(a, table_dtype, st);
}

extern "C" int smlm_quantize_q4(const float* table, int64_t rows, int64_t d, uint8_t* packed, void* scales_f16,
                                void* stream) {
    SMLM_CHECK_ARG(rows >= 0 && d >= 0 && d % 2 == 0 && d < (1 << 30), "quantize_q4: width must be even");
    if (rows == 0 || d == 0) return SMLM_OK;
    SMLM_CHECK_ARG(table && packed && scales_f16, "quantize_q4: null pointer");
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 16));
    quantize_q4_kernel<<<blocks, 256, 0, as_stream(stream)>>>(table, rows, (int)d, packed,
                                                              static_cast<uint16_t*>(scales_f16));
    SMLM_LAUNCHED("quantize_q4_kernel");
    return SMLM_OK;
}

extern "C" size_t smlm_bag_backward_workspace(int64_t n, int64_t k, int64_t rows, int64_t d) {
    if (n <= 0 || k <= 0) return 0;
    BackwardPlan p = plan_backward(n, k, rows);
    BackwardBufs b;
    return layout_backward(p, d, nullptr, &b);
}

namespace smlm {
// Both backward entry points: indices int64 / int32, table rows [row_base, row_base + rows) (skip_foreign: other
// rows are another shard's, skipped silently; else flagged).
static int backward_impl(const char* fn, const void* grad_out, int grad_dtype, const void* indices, int idx32,
                         int64_t row_base, int skip_foreign, const void* weights, int weights_dtype,
                         const void* table, int table_dtype, float* acc, uint8_t* touched, float* row_sqnorm,
                         int flags, float* gw, int64_t n, int64_t k, int64_t rows, int64_t d, void* workspace,
                         size_t workspace_bytes, int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && k >= 0 && rows >= 0 && d >= 0, "%s: negative size", fn);
    SMLM_CHECK_ARG(table_dtype == SMLM_F32 || table_dtype == SMLM_BF16, "%s: table must be fp32 or bf16", fn);
    SMLM_CHECK_ARG(weights_dtype == SMLM_F32 || weights_dtype == SMLM_BF16, "%s: weights must be fp32 or bf16", fn);
    SMLM_CHECK_ARG(grad_dtype == SMLM_F32 || grad_dtype == SMLM_BF16, "%s: grad_out must be fp32 or bf16", fn);
    SMLM_CHECK_ARG(n * k < (int64_t)0x7fffffff, "%s: n * k must be below 2^31", fn);
    SMLM_CHECK_ARG(rows < (int64_t)0xffffffff, "%s: rows must be below 2^32 - 1", fn);
    SMLM_CHECK_ARG(d <= SMLM_MAX_ROW_WIDTH, "%s: rows of %lld values are wider than the supported %d", fn,
                   (long long)d, SMLM_MAX_ROW_WIDTH);
    SMLM_CHECK_ARG((flags & ~(SMLM_BWD_FIRST_TOUCH_WRITES | SMLM_BWD_DEFER_ROWS)) == 0, "%s: unknown flags %d", fn,
                   flags);
    SMLM_CHECK_ARG(!(flags & SMLM_BWD_FIRST_TOUCH_WRITES) || touched != nullptr,
                   "%s: first-touch writes need the touched mask", fn);
    const bool defer = (flags & SMLM_BWD_DEFER_ROWS) != 0;
    SMLM_CHECK_ARG(!defer || (touched && row_sqnorm && (flags & SMLM_BWD_FIRST_TOUCH_WRITES)),
                   "%s: deferred row sums need first-touch writes, the touched mask and the row norms", fn);
    SMLM_CHECK_ARG(!defer || (d % 4 == 0 && d <= 512 &&
                              reinterpret_cast<uintptr_t>(grad_out) % (grad_dtype == SMLM_F32 ? 16 : 8) == 0),
                   "%s: deferred row sums need d %% 4 == 0, d <= 512 and an aligned grad_out", fn);
    if (n == 0 || k == 0) return SMLM_OK;
    SMLM_CHECK_ARG(grad_out && indices && weights && (table || !gw) && (gw || acc || defer), "%s: null pointer", fn);
    if (d == 0 && gw) {
        SMLM_CUDA(cudaMemsetAsync(gw, 0, sizeof(float) * n * k, as_stream(stream)));
    }
    BackwardPlan p = plan_backward(n, k, rows);
    BackwardBufs bb;
    const size_t need = layout_backward(p, d, nullptr, &bb);
    if (workspace == nullptr || workspace_bytes < need) {
        set_error("%s: workspace too small (%zu < %zu)", fn, workspace_bytes, need);
        return SMLM_ERR_WORKSPACE;
    }
    layout_backward(p, d, workspace, &bb);
    {
        // the weight gradient alone (no accumulator, no deferred rows): the gather-shaped kernel, no sort
        const uintptr_t tp = reinterpret_cast<uintptr_t>(table), gp = reinterpret_cast<uintptr_t>(grad_out);
        if (!defer && acc == nullptr && gw && d > 0 && d <= 512 && d % 4 == 0 &&
            gp % (grad_dtype == SMLM_F32 ? 16 : 8) == 0 && tp % (table_dtype == SMLM_F32 ? 16 : 8) == 0) {
            GwArgs ga{grad_out, indices, idx32, row_base, table, gw, n, rows, (int)k, (int)d};
            cudaStream_t s0 = as_stream(stream);
            if (table_dtype == SMLM_F32) {
                if (grad_dtype == SMLM_F32) launch_gw<float, float>(ga, s0);
                else launch_gw<float, __nv_bfloat16>(ga, s0);
            } else {
                if (grad_dtype == SMLM_F32) launch_gw<__nv_bfloat16, float>(ga, s0);
                else launch_gw<__nv_bfloat16, __nv_bfloat16>(ga, s0);
            }
            SMLM_LAUNCHED("bb_gw_kernel");
            return SMLM_OK;
        }
    }
    uint32_t *keys_in = bb.keys_in, *keys_out = bb.keys_out, *pos_in = bb.pos_in, *pos_out = bb.pos_out;
    void* sort_tmp = bb.sort_tmp;
    float *carry_head = bb.carry_head, *carry_tail = bb.carry_tail;
    int* chunk_flags = bb.flags;
    cudaStream_t st = as_stream(stream);
    const int kb = (int)std::max<int64_t>(1, std::min<int64_t>((p.m + 255) / 256, (int64_t)sm_count() * 8));
    bb_keys_kernel<<<kb, 256, 0, st>>>(indices, idx32, row_base, skip_foreign, p.m, rows, keys_in, pos_in, status);
    SMLM_LAUNCHED("bb_keys_kernel");
    size_t sort_bytes = p.sort_bytes;
    SMLM_CUDA(cub::DeviceRadixSort::SortPairs(sort_tmp, sort_bytes, keys_in, keys_out, pos_in, pos_out, (int)p.m, 0,
                                              std::max(p.end_bit, 1), st));
    if (d == 0) return SMLM_OK;
    SegArgs a{keys_out, pos_out, grad_out, grad_dtype, weights, weights_dtype, table, acc, touched, gw, carry_head,
              carry_tail, chunk_flags, row_sqnorm, (flags & SMLM_BWD_FIRST_TOUCH_WRITES) ? 1 : 0, p.m, rows, (int)k,
              (int)d, p.P, p.chunks};
    const uintptr_t tp = reinterpret_cast<uintptr_t>(table);
    const uintptr_t gp = reinterpret_cast<uintptr_t>(grad_out);
    const uintptr_t ap = reinterpret_cast<uintptr_t>(acc);
    const bool vec = d % 4 == 0 && gp % (grad_dtype == SMLM_F32 ? 16 : 8) == 0 && ap % 16 == 0 &&
                     tp % (table_dtype == SMLM_F32 ? 16 : 8) == 0;
    if (gw && vec && d <= 512) {
        // the weight gradient by its own gather-shaped kernel; the segment pass then sums rows only
        GwArgs ga{grad_out, indices, idx32, row_base, table, gw, n, rows, (int)k, (int)d};
        if (table_dtype == SMLM_F32) {
            if (grad_dtype == SMLM_F32) launch_gw<float, float>(ga, st);
            else launch_gw<float, __nv_bfloat16>(ga, st);
        } else {
            if (grad_dtype == SMLM_F32) launch_gw<__nv_bfloat16, float>(ga, st);
            else launch_gw<__nv_bfloat16, __nv_bfloat16>(ga, st);
        }
        SMLM_LAUNCHED("bb_gw_kernel");
        a.gw = nullptr;
        if (acc == nullptr && !defer) return SMLM_OK;
    }
    if (defer) {
        SMLM_CHECK_ARG(a.gw == nullptr, "%s: deferred row sums need an aligned table for the weight gradient", fn);
        const RowAdam none{};
        return grad_dtype == SMLM_F32 ? launch_rows_mode<float, ROWS_NORM>(a, none, st)
                                      : launch_rows_mode<__nv_bfloat16, ROWS_NORM>(a, none, st);
    }
    if (table_dtype == SMLM_F32) return vec ? launch_segment_g<float, 4>(a, st) : launch_segment_g<float, 1>(a, st);
    return vec ? launch_segment_g<__nv_bfloat16, 4>(a, st) : launch_segment_g<__nv_bfloat16, 1>(a, st);
}
}  // namespace smlm

extern "C" int smlm_bag_backward_rows(const void* grad_out, int grad_dtype, const int64_t* indices,
                                      const void* weights, int weights_dtype, const void* table, int table_dtype,
                                      float* acc, uint8_t* touched, float* row_sqnorm, int flags, float* gw,
                                      int64_t n, int64_t k, int64_t rows, int64_t d, void* workspace,
                                      size_t workspace_bytes, int* status, void* stream) {
    return backward_impl("bag_backward_rows", grad_out, grad_dtype, indices, 0, 0, 0, weights, weights_dtype, table,
                         table_dtype, acc, touched, row_sqnorm, flags, gw, n, k, rows, d, workspace, workspace_bytes,
                         status, stream);
}

extern "C" int smlm_shard_bag_backward_rows(const void* grad_out, int grad_dtype, const void* indices,
                                            int index_dtype, int64_t row_base, const void* weights,
                                            int weights_dtype, const void* table_shard, int table_dtype, float* acc,
                                            uint8_t* touched, float* row_sqnorm, int flags, float* gw, int64_t n,
                                            int64_t k, int64_t shard_rows, int64_t d, void* workspace,
                                            size_t workspace_bytes, int* status, void* stream) {
    SMLM_CHECK_ARG(index_dtype == SMLM_I32 || index_dtype == SMLM_I64, "shard_bag_backward_rows: int32 or int64 indices");
    SMLM_CHECK_ARG(row_base >= 0, "shard_bag_backward_rows: negative row base");
    return backward_impl("shard_bag_backward_rows", grad_out, grad_dtype, indices, index_dtype == SMLM_I32, row_base,
                         1, weights, weights_dtype, table_shard, table_dtype, acc, touched, row_sqnorm, flags, gw, n,
                         k, shard_rows, d, workspace, workspace_bytes, status, stream);
}

namespace smlm {
// The sorted (row, position) pairs a deferred backward left in its workspace, for the passes that finish it.
static int deferred_args(const char* fn, const void* grad_out, int grad_dtype, const void* weights, int weights_dtype,
                         int64_t n, int64_t k, int64_t rows, int64_t d, void* workspace, size_t workspace_bytes,
                         SegArgs* a) {
    SMLM_CHECK_ARG(n >= 0 && k >= 0 && rows >= 0 && d % 4 == 0 && d > 0 && d <= 512, "%s: bad sizes", fn);
    SMLM_CHECK_ARG(weights_dtype == SMLM_F32 || weights_dtype == SMLM_BF16, "%s: weights must be fp32 or bf16", fn);
    SMLM_CHECK_ARG(grad_dtype == SMLM_F32 || grad_dtype == SMLM_BF16, "%s: grad_out must be fp32 or bf16", fn);
    SMLM_CHECK_ARG(n * k < (int64_t)0x7fffffff && rows < (int64_t)0xffffffff, "%s: size too large", fn);
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(grad_out) % (grad_dtype == SMLM_F32 ? 16 : 8) == 0,
                   "%s: grad_out must be aligned", fn);
    if (n == 0 || k == 0) return SMLM_OK;  // an empty backward left nothing to sum (the callers return here too)
    BackwardPlan p = plan_backward(n, k, rows);
    BackwardBufs bb;
    const size_t need = layout_backward(p, d, nullptr, &bb);
    if (workspace == nullptr || workspace_bytes < need) {
        set_error("%s: workspace too small (%zu < %zu)", fn, workspace_bytes, need);
        return SMLM_ERR_WORKSPACE;
    }
    layout_backward(p, d, workspace, &bb);
    *a = SegArgs{bb.keys_out, bb.pos_out, grad_out, grad_dtype, weights, weights_dtype, nullptr, nullptr, nullptr,
                 nullptr, bb.carry_head, bb.carry_tail, bb.flags, nullptr, 1, p.m, rows, (int)k, (int)d, p.P,
                 p.chunks, 1};
    return SMLM_OK;
}
}  // namespace smlm

extern "C" int smlm_bag_rows_materialize(const void* grad_out, int grad_dtype, const void* weights, int weights_dtype,
                                         float* acc, int64_t n, int64_t k, int64_t rows, int64_t d, void* workspace,
                                         size_t workspace_bytes, void* stream) {
    SegArgs a;
    int rc = deferred_args("bag_rows_materialize", grad_out, grad_dtype, weights, weights_dtype, n, k, rows, d,
                           workspace, workspace_bytes, &a);
    if (rc != SMLM_OK || n == 0 || k == 0) return rc;
    SMLM_CHECK_ARG(acc && reinterpret_cast<uintptr_t>(acc) % 16 == 0, "bag_rows_materialize: acc must be aligned");
    a.acc = acc;
    const RowAdam none{};
    cudaStream_t st = as_stream(stream);
    return grad_dtype == SMLM_F32 ? launch_rows_mode<float, ROWS_WRITE>(a, none, st)
                                  : launch_rows_mode<__nv_bfloat16, ROWS_WRITE>(a, none, st);
}

namespace smlm {
static int lazy_adam_deferred_impl(float* param, float* exp_avg, float* exp_avg_sq, uint8_t* touched,
                                   const void* grad_out, int grad_dtype, const void* weights, int weights_dtype,
                                   const float* grad_scale_dev, float grad_scale, int64_t n, int64_t k, int64_t rows,
                                   int64_t d, AdamScalars sc, const float* scalars_dev, void* value_copy,
                                   int copy_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    SegArgs a;
    int rc = deferred_args("lazy_adam_deferred_step", grad_out, grad_dtype, weights, weights_dtype, n, k, rows, d,
                           workspace, workspace_bytes, &a);
    if (rc != SMLM_OK || n == 0 || k == 0) return rc;
    SMLM_CHECK_ARG(param && exp_avg && exp_avg_sq && touched, "lazy_adam_deferred_step: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(param) % 16 == 0 && reinterpret_cast<uintptr_t>(exp_avg) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(exp_avg_sq) % 16 == 0 &&
                       (value_copy == nullptr || reinterpret_cast<uintptr_t>(value_copy) % 16 == 0),
                   "lazy_adam_deferred_step: tables must be 16-byte aligned");
    SMLM_CHECK_ARG(value_copy == nullptr || copy_dtype == SMLM_F32 || copy_dtype == SMLM_BF16,
                   "lazy_adam_deferred_step: value copy must be fp32 or bf16");
    a.touched = touched;
    RowAdam ad{param, exp_avg, exp_avg_sq, grad_scale_dev, grad_scale, sc, value_copy, copy_dtype};
    ad.s_dev = scalars_dev;
    cudaStream_t st = as_stream(stream);
    return grad_dtype == SMLM_F32 ? launch_rows_mode<float, ROWS_ADAM>(a, ad, st)
                                  : launch_rows_mode<__nv_bfloat16, ROWS_ADAM>(a, ad, st);
}
}  // namespace smlm

extern "C" int smlm_lazy_adam_deferred_step(float* param, float* exp_avg, float* exp_avg_sq, uint8_t* touched,
                                            const void* grad_out, int grad_dtype, const void* weights,
                                            int weights_dtype, const float* grad_scale_dev, float grad_scale,
                                            int64_t n, int64_t k, int64_t rows, int64_t d, float one_minus_b1, float b2,
                                            float one_minus_b2, float bc2_sqrt, float eps, float neg_step_size,
                                            void* value_copy, int copy_dtype, void* workspace, size_t workspace_bytes,
                                            void* stream) {
    return smlm::lazy_adam_deferred_impl(param, exp_avg, exp_avg_sq, touched, grad_out, grad_dtype, weights,
                                         weights_dtype, grad_scale_dev, grad_scale, n, k, rows, d,
                                         smlm::AdamScalars{one_minus_b1, b2, one_minus_b2, bc2_sqrt, eps,
                                                           neg_step_size},
                                         nullptr, value_copy, copy_dtype, workspace, workspace_bytes, stream);
}

extern "C" int smlm_lazy_adam_deferred_step_dev(float* param, float* exp_avg, float* exp_avg_sq, uint8_t* touched,
                                                const void* grad_out, int grad_dtype, const void* weights,
                                                int weights_dtype, const float* grad_scale_dev, float grad_scale,
                                                int64_t n, int64_t k, int64_t rows, int64_t d,
                                                const float* scalars_dev, void* value_copy, int copy_dtype,
                                                void* workspace, size_t workspace_bytes, void* stream) {
    SMLM_CHECK_ARG(scalars_dev != nullptr, "lazy_adam_deferred_step_dev: null scalars");
    return smlm::lazy_adam_deferred_impl(param, exp_avg, exp_avg_sq, touched, grad_out, grad_dtype, weights,
                                         weights_dtype, grad_scale_dev, grad_scale, n, k, rows, d,
                                         smlm::AdamScalars{}, scalars_dev, value_copy, copy_dtype, workspace,
                                         workspace_bytes, stream);
}

extern "C" int smlm_rowwise_deferred_step(float* param, uint8_t* touched, float* v, int32_t* count,
                                          const void* grad_out, int grad_dtype, const void* weights,
                                          int weights_dtype, const float* grad_scale_dev, float grad_scale,
                                          int64_t n, int64_t k, int64_t rows, int64_t d, int kind, float b2,
                                          float eps, float lr, void* workspace, size_t workspace_bytes,
                                          void* stream) {
    SegArgs a;
    int rc = deferred_args("rowwise_deferred_step", grad_out, grad_dtype, weights, weights_dtype, n, k, rows, d,
                           workspace, workspace_bytes, &a);
    if (rc != SMLM_OK || n == 0 || k == 0) return rc;
    SMLM_CHECK_ARG(kind == SMLM_ROWRMS || kind == SMLM_ROWADAGRAD, "rowwise_deferred_step: unknown kind %d", kind);
    SMLM_CHECK_ARG(param && touched && v && (count || kind == SMLM_ROWADAGRAD), "rowwise_deferred_step: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(param) % 16 == 0, "rowwise_deferred_step: table must be 16-byte aligned");
    a.touched = touched;
    RowAdam ad{};
    ad.p = param;
    ad.scale_dev = grad_scale_dev;
    ad.scale = grad_scale;
    ad.row_v = v;
    ad.row_count = count;
    ad.rw_kind = kind;
    ad.rw_b2 = b2;
    ad.rw_eps = eps;
    ad.rw_lr = lr;
    cudaStream_t st = as_stream(stream);
    return grad_dtype == SMLM_F32 ? launch_rows_mode<float, ROWS_ROWWISE>(a, ad, st)
                                  : launch_rows_mode<__nv_bfloat16, ROWS_ROWWISE>(a, ad, st);
}
