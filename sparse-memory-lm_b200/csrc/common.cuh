// Shared device/host helpers for the PKM layer kernels (sm_100a only).
//
// Every kernel in this library is launched on the caller's stream, allocates nothing (scratch comes in
// through a workspace pointer whose size the matching *_workspace query returns), and never traps: index
// range violations set a bit in a caller-provided device status word and the offending lookup is skipped.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include <algorithm>
#include <type_traits>

#include "../../include/smlm_b200.h"

#if !defined(__CUDA_ARCH__) || __CUDA_ARCH__ >= 1000
#else
#error "this library is built for sm_100a only"
#endif

namespace smlm {

// ------------------------------------------------------------------------------------------------ host side
// Thread-local last-error message, read through smlm_last_error().
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

#define SMLM_CHECK_ARG(cond, ...)                 \
    do {                                          \
        if (!(cond)) {                            \
            ::smlm::set_error(__VA_ARGS__);       \
            return SMLM_ERR_INVALID;              \
        }                                         \
    } while (0)

#define SMLM_CUDA(call)                                              \
    do {                                                             \
        cudaError_t _e = (call);                                     \
        if (_e != cudaSuccess) return ::smlm::cuda_status(_e, #call); \
    } while (0)

#define SMLM_LAUNCHED(what)                                          \
    do {                                                             \
        cudaError_t _e = cudaGetLastError();                         \
        if (_e != cudaSuccess) return ::smlm::cuda_status(_e, what); \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int sm_count();

// Bump allocator over a caller-provided workspace; every slice is 256-byte aligned.
struct Workspace {
    char* base;
    size_t size;
    size_t used = 0;
    Workspace(void* b, size_t s) : base(static_cast<char*>(b)), size(s) {}
    template <typename T>
    T* take(size_t count) {
        size_t off = (used + 255) & ~size_t(255);
        used = off + count * sizeof(T);
        return reinterpret_cast<T*>(base + off);
    }
    bool ok() const { return used <= size; }
};
// The same carve-up without a base pointer, for the size queries.
struct WorkspaceSize {
    size_t used = 0;
    template <typename T>
    void take(size_t count) { used = ((used + 255) & ~size_t(255)) + count * sizeof(T); }
};

// ---------------------------------------------------------------------------------------------- device side
constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// fp32 -> bf16 bits, round to nearest even (PyTorch's c10::BFloat16 rounding for finite values).
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0u;  // NaN
    return (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ float round_bf16(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }
// silu(p) = p * sigmoid(p) as the swilu product's factor, rounded to bf16 as the reference's autocast computes it
__device__ __forceinline__ float silu_bf16(float p) { return round_bf16(p / (1.0f + expf(-p))); }

// Order-preserving unsigned codes: a larger code means a larger value; -0 is mapped onto +0 so that the two
// zeros tie (and the tie goes to the lower index, as for any other equal scores).
__device__ __forceinline__ uint32_t order_code16(uint32_t b) {
    b &= 0xffffu;
    if (b == 0x8000u) b = 0;
    return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}
__device__ __forceinline__ uint32_t decode_code16(uint32_t c) {
    return (c & 0x8000u) ? (c ^ 0x8000u) : (~c & 0xffffu);
}
__device__ __forceinline__ uint32_t order_code32(uint32_t u) {
    if (u == 0x80000000u) u = 0;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint32_t decode_code32(uint32_t c) {
    return (c & 0x80000000u) ? (c ^ 0x80000000u) : ~c;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

__device__ __forceinline__ void flag(int* status, int bit) {
    if (status) atomicOr(status, bit);
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

// Lazy Adam update of one element in the reference C loop's order (host_rows.c:69-76), every operation rounded
// on its own: the one definition used by every Adam kernel of the library.
struct AdamScalars {
    float one_minus_b1, b2, one_minus_b2, bc2_sqrt, eps, neg_step;
};
__device__ __forceinline__ void adam_update(const AdamScalars& a, float scale, float& p, float& m, float& v, float g) {
    const float gk = __fmul_rn(g, scale);
    const float mk = __fadd_rn(m, __fmul_rn(a.one_minus_b1, __fsub_rn(gk, m)));
    const float vk = __fadd_rn(__fmul_rn(v, a.b2), __fmul_rn(__fmul_rn(a.one_minus_b2, gk), gk));
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vk), a.bc2_sqrt), a.eps);
    p = __fadd_rn(p, __fmul_rn(a.neg_step, __fdiv_rn(mk, denom)));
    m = mk;
    v = vk;
}

// Row-wise optimizer state update of row r from q = mean of the row's squared gradient (the reference C loop's
// formulas and rounding, host_rows.c:84-117; fp32 state, the bias correction in double): returns the step size
// lr / denom; lane 0 writes the row's state (call with the whole warp, after q is reduced). The one definition used
// by every row-wise kernel of the library.
__device__ __forceinline__ float rowwise_state_step(int kind, float b2, float eps, float lr, float* v, int32_t* count,
                                                    int64_t r, double q, int lane) {
    float denom;
    if (kind == SMLM_ROWRMS) {
        const float one_minus_b2 = __fsub_rn(1.0f, b2);
        const float vr = __fadd_rn(__fmul_rn(b2, v[r]), __fmul_rn(one_minus_b2, (float)q));
        const int32_t cnt = count[r] + 1;
        denom = __fadd_rn(__fsqrt_rn((float)((double)vr / (1.0 - pow((double)b2, (double)cnt)))), eps);
        __syncwarp();
        if (lane == 0) {
            v[r] = vr;
            count[r] = cnt;
        }
    } else {
        const float vr = __fadd_rn(v[r], (float)q);
        denom = __fadd_rn(__fsqrt_rn(vr), eps);
        __syncwarp();
        if (lane == 0) v[r] = vr;
    }
    return __fdiv_rn(lr, denom);
}

// One row of the row-wise step, by one warp: q = mean of (g * sc)^2, summed in double over each lane's groups of VEC
// consecutive columns (lane * VEC + 32 * VEC * k, in column order) and then across the warp; the state step; then
// dst[c] = src[c] - step * (g[c] * sc), and g's row set to 0 when zero_g. VEC == 4 moves the rows with 16-byte
// accesses (g, src, dst 16-byte aligned, d % 4 == 0), which matters most when a row lives in mapped host memory
// (one request per 16 bytes instead of four); with NC > 0 (d <= 128 * NC) each lane keeps its NC float4 groups of g
// in registers between the two passes, so g is read once. Same operations in the same order for every VEC / NC.
template <int VEC, int NC>
__device__ __forceinline__ void rowwise_row(const float* g, bool zero_g, const float* src, float* dst, int d, float sc,
                                            int kind, float b2, float eps, float lr, float* v, int32_t* count,
                                            int64_t r, int lane) {
    double q = 0.0;
    if constexpr (VEC == 4) {
        float4 gc[NC > 0 ? NC : 1];
        if constexpr (NC > 0) {
#pragma unroll
            for (int k = 0; k < NC; k++) {
                const int c = lane * 4 + 128 * k;
                if (c < d) gc[k] = *reinterpret_cast<const float4*>(g + c);
            }
        }
        auto sq = [&](const float4 x) {
            const float g0 = __fmul_rn(x.x, sc), g1 = __fmul_rn(x.y, sc), g2 = __fmul_rn(x.z, sc),
                        g3 = __fmul_rn(x.w, sc);
            q = fma((double)g0, (double)g0, q);
            q = fma((double)g1, (double)g1, q);
            q = fma((double)g2, (double)g2, q);
            q = fma((double)g3, (double)g3, q);
        };
        if constexpr (NC > 0) {
#pragma unroll
            for (int k = 0; k < NC; k++)
                if (lane * 4 + 128 * k < d) sq(gc[k]);
        } else {
            for (int c = lane * 4; c < d; c += 128) sq(*reinterpret_cast<const float4*>(g + c));
        }
        q = warp_sum_d(q) / (double)d;
        const float step = rowwise_state_step(kind, b2, eps, lr, v, count, r, q, lane);
        auto upd = [&](const int c, const float4 x) {
            float4 p = *reinterpret_cast<const float4*>(src + c);
            p.x = __fsub_rn(p.x, __fmul_rn(step, __fmul_rn(x.x, sc)));
            p.y = __fsub_rn(p.y, __fmul_rn(step, __fmul_rn(x.y, sc)));
            p.z = __fsub_rn(p.z, __fmul_rn(step, __fmul_rn(x.z, sc)));
            p.w = __fsub_rn(p.w, __fmul_rn(step, __fmul_rn(x.w, sc)));
            *reinterpret_cast<float4*>(dst + c) = p;
            if (zero_g) *reinterpret_cast<float4*>(const_cast<float*>(g) + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        };
        if constexpr (NC > 0) {
#pragma unroll
            for (int k = 0; k < NC; k++) {
                const int c = lane * 4 + 128 * k;
                if (c < d) upd(c, gc[k]);
            }
        } else {
            for (int c = lane * 4; c < d; c += 128) upd(c, *reinterpret_cast<const float4*>(g + c));
        }
    } else {
        for (int c = lane; c < d; c += 32) {
            const float gk = __fmul_rn(g[c], sc);
            q = fma((double)gk, (double)gk, q);
        }
        q = warp_sum_d(q) / (double)d;
        const float step = rowwise_state_step(kind, b2, eps, lr, v, count, r, q, lane);
        for (int c = lane; c < d; c += 32) {
            const float gk = __fmul_rn(g[c], sc);
            dst[c] = __fsub_rn(src[c], __fmul_rn(step, gk));
            if (zero_g) const_cast<float*>(g)[c] = 0.f;
        }
    }
}

// The register groups rowwise_row keeps per lane for width d (0: d > 512, g read twice).
inline int rowwise_groups(int64_t d) { return d <= 128 ? 1 : d <= 256 ? 2 : d <= 384 ? 3 : d <= 512 ? 4 : 0; }

// Vector loads of VEC elements (fp32 or bf16) widened to fp32 (16-byte / 8-byte loads for VEC == 4).
template <typename T>
struct Elt;
template <>
struct Elt<float> {
    template <int VEC>
    __device__ __forceinline__ static void load(const float* p, float (&v)[VEC]) {
        if constexpr (VEC == 4) {
            float4 x = __ldg(reinterpret_cast<const float4*>(p));
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
#pragma unroll
            for (int i = 0; i < VEC; i++) v[i] = __ldg(p + i);
        }
    }
};
template <>
struct Elt<__nv_bfloat16> {
    template <int VEC>
    __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&v)[VEC]) {
        if constexpr (VEC == 4) {
            uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
            v[0] = bf16_bits_to_f32(x.x & 0xffffu);
            v[1] = bf16_bits_to_f32(x.x >> 16);
            v[2] = bf16_bits_to_f32(x.y & 0xffffu);
            v[3] = bf16_bits_to_f32(x.y >> 16);
        } else {
            const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
            for (int i = 0; i < VEC; i++) v[i] = bf16_bits_to_f32(__ldg(q + i));
        }
    }
};


}  // namespace smlm
