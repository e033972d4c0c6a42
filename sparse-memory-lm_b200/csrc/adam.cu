// Row-sparse optimizer steps over the touched rows only: lazy Adam (fp32 moments), the row-wise rowrms /
// rowadagrad variant, and the accumulator norm used for clipping.
//
// Each entry first compacts the touched mask into an ascending list of row ids plus its length, both in the
// workspace (cub::DeviceSelect::Flagged; ordered, deterministic); the update kernels are persistent grids that
// read the length from device memory, so nothing syncs with the host. One warp per row, 16-byte vectors.
#include <cub/device/device_select.cuh>
#include <cub/iterator/counting_input_iterator.cuh>

#include "common.cuh"

namespace smlm {

struct TouchedBufs {
    int32_t* list;
    int32_t* count;
    void* tmp;
    size_t tmp_bytes;
    double* partials;
};

constexpr int PARTIALS = 8192;  // per-warp partial sums of the norm kernel (fixed: deterministic order)

static size_t select_tmp_bytes(int64_t rows) {
    size_t bytes = 0;
    cub::DeviceSelect::Flagged(nullptr, bytes, cub::CountingInputIterator<int32_t>(0), (const uint8_t*)nullptr,
                               (int32_t*)nullptr, (int32_t*)nullptr, (int)std::max<int64_t>(rows, 1));
    return bytes;
}

static size_t layout_touched(int64_t rows, void* base, TouchedBufs* b) {
    size_t off = 0;
    char* c = static_cast<char*>(base);
    auto take = [&](size_t bytes) -> void* {
        off = (off + 255) & ~size_t(255);
        void* ptr = c ? c + off : nullptr;
        off += bytes;
        return ptr;
    };
    b->list = static_cast<int32_t*>(take(sizeof(int32_t) * std::max<int64_t>(rows, 1)));
    b->count = static_cast<int32_t*>(take(sizeof(int32_t) * 4));
    b->tmp_bytes = select_tmp_bytes(rows);
    b->tmp = take(b->tmp_bytes);
    b->partials = static_cast<double*>(take(sizeof(double) * PARTIALS));
    return off;
}

static int compact_touched(const uint8_t* touched, int64_t rows, void* workspace, size_t workspace_bytes,
                           TouchedBufs* b, cudaStream_t st) {
    const size_t need = layout_touched(rows, nullptr, b);
    if (workspace == nullptr || workspace_bytes < need) {
        set_error("touched-row workspace too small (%zu < %zu)", workspace_bytes, need);
        return SMLM_ERR_WORKSPACE;
    }
    layout_touched(rows, workspace, b);
    size_t tmp = b->tmp_bytes;
    SMLM_CUDA(cub::DeviceSelect::Flagged(b->tmp, tmp, cub::CountingInputIterator<int32_t>(0), touched, b->list,
                                         b->count, (int)rows, st));
    return SMLM_OK;
}

static int persistent_blocks(int warps_per_block, int per_sm) {
    (void)warps_per_block;
    return sm_count() * per_sm;
}

// ------------------------------------------------------------------------------------------------ lazy Adam
struct AdamArgs {
    float *p, *m, *v, *acc;
    uint8_t* touched;
    const int32_t* list;
    const int32_t* count;
    const float* scale_dev;
    float scale;
    int d;
    float one_minus_b1, b2, one_minus_b2, bc2_sqrt, eps, neg_step;
    void* copy;
    int copy_dtype;
    int keep_acc;        // leave the consumed accumulator rows as they are (they count as zero once untouched)
    const float* s_dev;  // the six scalars above from device memory instead (a step captured in a CUDA graph)
};

// Element update in the reference C loop's order (host_rows.c:69-76), every operation rounded on its own.
__device__ __forceinline__ void adam_elem(const AdamScalars& sc, float scale, float& p, float& m, float& v, float g) {
    adam_update(sc, scale, p, m, v, g);
}

template <int VEC>
__global__ void __launch_bounds__(256) lazy_adam_kernel(AdamArgs a) {
    const int lane = lane_id();
    const int n = *a.count;
    const float scale = a.scale_dev ? *a.scale_dev : a.scale;
    const AdamScalars sc = a.s_dev ? AdamScalars{a.s_dev[0], a.s_dev[1], a.s_dev[2], a.s_dev[3], a.s_dev[4], a.s_dev[5]}
                                   : AdamScalars{a.one_minus_b1, a.b2, a.one_minus_b2, a.bc2_sqrt, a.eps, a.neg_step};
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int64_t r = a.list[i];
        const int64_t base = r * a.d;
        if constexpr (VEC == 4) {
#pragma unroll 3
            for (int c = lane * 4; c < a.d; c += 128) {
                float4 p = *reinterpret_cast<float4*>(a.p + base + c);
                float4 m = *reinterpret_cast<float4*>(a.m + base + c);
                float4 v = *reinterpret_cast<float4*>(a.v + base + c);
                const float4 g = *reinterpret_cast<float4*>(a.acc + base + c);
                adam_elem(sc, scale, p.x, m.x, v.x, g.x);
                adam_elem(sc, scale, p.y, m.y, v.y, g.y);
                adam_elem(sc, scale, p.z, m.z, v.z, g.z);
                adam_elem(sc, scale, p.w, m.w, v.w, g.w);
                *reinterpret_cast<float4*>(a.p + base + c) = p;
                *reinterpret_cast<float4*>(a.m + base + c) = m;
                *reinterpret_cast<float4*>(a.v + base + c) = v;
                if (!a.keep_acc) *reinterpret_cast<float4*>(a.acc + base + c) = make_float4(0.f, 0.f, 0.f, 0.f);
                if (a.copy) {
                    if (a.copy_dtype == SMLM_BF16) {
                        uint2 o;
                        o.x = f32_to_bf16_bits(p.x) | (f32_to_bf16_bits(p.y) << 16);
                        o.y = f32_to_bf16_bits(p.z) | (f32_to_bf16_bits(p.w) << 16);
                        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.copy) + base + c) = o;
                    } else {
                        *reinterpret_cast<float4*>(static_cast<float*>(a.copy) + base + c) = p;
                    }
                }
            }
        } else {
            for (int c = lane; c < a.d; c += 32) {
                float p = a.p[base + c], m = a.m[base + c], v = a.v[base + c];
                adam_elem(sc, scale, p, m, v, a.acc[base + c]);
                a.p[base + c] = p;
                a.m[base + c] = m;
                a.v[base + c] = v;
                if (!a.keep_acc) a.acc[base + c] = 0.f;
                if (a.copy) {
                    if (a.copy_dtype == SMLM_BF16) static_cast<uint16_t*>(a.copy)[base + c] = (uint16_t)f32_to_bf16_bits(p);
                    else static_cast<float*>(a.copy)[base + c] = p;
                }
            }
        }
        __syncwarp();
        if (lane == 0) a.touched[r] = 0;
    }
}

// ----------------------------------------------------------------------------------- lazy Adam, compact state
// bf16 moments, or int8 codes with one fp32 scale per row: m = sign * (code / 127)^2 * m_scale (signed square
// root), v = ((code / 255) * v_scale)^4 (unsigned fourth root). The update runs in fp32 on the decoded moments;
// only the stored state is rounded. Operation order and rounding of the reference's compact kernel
// (kernels.py:445-495): every operation rounded on its own, stores rounded to nearest even, a positive second
// moment never gets a zero code.
struct LowArgs {
    float *p, *acc;
    void *m, *v;
    float *m_scale, *v_scale;
    uint8_t* touched;
    const int32_t* list;
    const int32_t* count;
    const float* scale_dev;
    float scale;
    int d;
    float b1, b2, one_minus_b1, one_minus_b2, eps, step_size, bc2_sqrt;
    void* copy;
    int copy_dtype;
    int keep_acc;
};

__device__ __forceinline__ float sign_one(float x) { return x < 0.f ? -1.f : 1.f; }

template <bool INT8>
__device__ __forceinline__ void low_load(const LowArgs& a, int64_t i, float ms, float vs, float& m, float& v) {
    if constexpr (INT8) {
        const float mc = __fdiv_rn((float)static_cast<const int8_t*>(a.m)[i], 127.f);
        m = __fmul_rn(__fmul_rn(__fmul_rn(sign_one(mc), mc), mc), ms);
        const float vc = __fmul_rn(__fdiv_rn((float)static_cast<const uint8_t*>(a.v)[i], 255.f), vs);
        v = __fmul_rn(vc, vc);
        v = __fmul_rn(v, v);
    } else {
        m = bf16_bits_to_f32(static_cast<const uint16_t*>(a.m)[i]);
        v = bf16_bits_to_f32(static_cast<const uint16_t*>(a.v)[i]);
    }
}

__device__ __forceinline__ void low_update(const LowArgs& a, float g, float& p, float& m, float& v) {
    m = __fadd_rn(__fmul_rn(a.b1, m), __fmul_rn(a.one_minus_b1, g));
    v = __fadd_rn(__fmul_rn(a.b2, v), __fmul_rn(__fmul_rn(a.one_minus_b2, g), g));
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), a.bc2_sqrt), a.eps);
    p = __fsub_rn(p, __fdiv_rn(__fmul_rn(a.step_size, m), denom));
}

__device__ __forceinline__ float fourth_root(float v) { return __fsqrt_rn(__fsqrt_rn(v)); }

template <bool INT8>
__device__ __forceinline__ void low_store(const LowArgs& a, int64_t i, float ms, float vs, float p, float m,
                                          float v) {
    a.p[i] = p;
    if constexpr (INT8) {
        float mq = __fsqrt_rn(__fdiv_rn(fabsf(m), ms > 0.f ? ms : 1.f));
        mq = rintf(fminf(fmaxf(__fmul_rn(__fmul_rn(sign_one(m), mq), 127.f), -127.f), 127.f));
        float vq = __fmul_rn(__fdiv_rn(fourth_root(v), vs > 0.f ? vs : 1.f), 255.f);
        vq = rintf(fminf(fmaxf(vq, 0.f), 255.f));
        vq = v > 0.f ? fmaxf(vq, 1.f) : 0.f;
        static_cast<int8_t*>(a.m)[i] = (int8_t)mq;
        static_cast<uint8_t*>(a.v)[i] = (uint8_t)vq;
    } else {
        static_cast<uint16_t*>(a.m)[i] = (uint16_t)f32_to_bf16_bits(m);
        static_cast<uint16_t*>(a.v)[i] = (uint16_t)f32_to_bf16_bits(v);
    }
    if (!a.keep_acc) a.acc[i] = 0.f;
    if (a.copy) {
        if (a.copy_dtype == SMLM_BF16) static_cast<uint16_t*>(a.copy)[i] = (uint16_t)f32_to_bf16_bits(p);
        else static_cast<float*>(a.copy)[i] = p;
    }
}

// One warp per touched row. NS > 0: the row (d <= 32 NS) stays in registers between the update and the int8
// encode, which needs the row maxima of the new moments. NS == 0 (any width): bf16 streams the row once; int8
// runs the update twice, first for the maxima, then to encode (same inputs, same results).
template <bool INT8, int NS>
__global__ void __launch_bounds__(256) lazy_adam_lowmem_kernel(LowArgs a) {
    const int lane = lane_id();
    const int n = *a.count;
    const float scale = a.scale_dev ? *a.scale_dev : a.scale;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int64_t r = a.list[i];
        const int64_t base = r * a.d;
        const float ms_old = INT8 ? a.m_scale[r] : 0.f, vs_old = INT8 ? a.v_scale[r] : 0.f;
        float ms = 0.f, vs = 0.f;
        if constexpr (NS > 0) {
            float p[NS], m[NS], v[NS];
#pragma unroll
            for (int s = 0; s < NS; s++) {
                const int c = lane + 32 * s;
                p[s] = m[s] = v[s] = 0.f;
                if (c < a.d) {
                    const float g = __fmul_rn(a.acc[base + c], scale);
                    low_load<INT8>(a, base + c, ms_old, vs_old, m[s], v[s]);
                    p[s] = a.p[base + c];
                    low_update(a, g, p[s], m[s], v[s]);
                    if (INT8) {
                        ms = fmaxf(ms, fabsf(m[s]));
                        vs = fmaxf(vs, fourth_root(v[s]));
                    }
                }
            }
            if (INT8) {
                ms = warp_max(ms);
                vs = warp_max(vs);
            }
#pragma unroll
            for (int s = 0; s < NS; s++) {
                const int c = lane + 32 * s;
                if (c < a.d) low_store<INT8>(a, base + c, ms, vs, p[s], m[s], v[s]);
            }
        } else {
            if (INT8) {
                for (int c = lane; c < a.d; c += 32) {
                    float p = a.p[base + c], m, v;
                    low_load<INT8>(a, base + c, ms_old, vs_old, m, v);
                    low_update(a, __fmul_rn(a.acc[base + c], scale), p, m, v);
                    ms = fmaxf(ms, fabsf(m));
                    vs = fmaxf(vs, fourth_root(v));
                }
                ms = warp_max(ms);
                vs = warp_max(vs);
            }
            __syncwarp();
            for (int c = lane; c < a.d; c += 32) {
                float p = a.p[base + c], m, v;
                low_load<INT8>(a, base + c, ms_old, vs_old, m, v);
                low_update(a, __fmul_rn(a.acc[base + c], scale), p, m, v);
                low_store<INT8>(a, base + c, ms, vs, p, m, v);
            }
        }
        __syncwarp();
        if (lane == 0) {
            if (INT8) {
                a.m_scale[r] = ms;
                a.v_scale[r] = vs;
            }
            a.touched[r] = 0;
        }
    }
}

// ------------------------------------------------------------------------------------------------ row-wise
struct RowArgs {
    float *p, *acc, *v;
    int32_t* count_state;
    uint8_t* touched;
    const int32_t* list;
    const int32_t* count;
    const float* scale_dev;
    float scale;
    int d, kind;
    float b2, eps, lr;
    int keep_acc;
};

// Formulas and rounding of the reference C loop (host_rows.c:84-117): q summed in double, row state in fp32.
template <int VEC, int NC>
__global__ void __launch_bounds__(256) rowwise_kernel(RowArgs a) {
    const int lane = lane_id();
    const int n = *a.count;
    const float scale = a.scale_dev ? *a.scale_dev : a.scale;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int64_t r = a.list[i];
        const int64_t base = r * a.d;
        rowwise_row<VEC, NC>(a.acc + base, !a.keep_acc, a.p + base, a.p + base, a.d, scale, a.kind, a.b2, a.eps,
                             a.lr, a.v, a.count_state, r, lane);
        __syncwarp();
        if (lane == 0) a.touched[r] = 0;
    }
}

// --------------------------------------------------------------------------------------------------- norm
// Pass 1: warp w sums the squares of rows list[w], list[w + W], ... (double); W = PARTIALS fixed, so the
// summation order does not depend on the device. Pass 2: one warp adds the PARTIALS in a fixed tree.
template <int VEC>
__global__ void __launch_bounds__(256) touched_sq_kernel(const float* acc, const int32_t* list, const int32_t* count,
                                                         int d, double* partials) {
    const int lane = lane_id();
    const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= PARTIALS) return;
    const int n = *count;
    double s = 0.0;
    for (int i = w; i < n; i += PARTIALS) {
        const int64_t base = (int64_t)list[i] * d;
        if constexpr (VEC == 4) {
#pragma unroll 3
            for (int c = lane * 4; c < d; c += 128) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(acc + base + c));
                s = fma((double)x.x, (double)x.x, s);
                s = fma((double)x.y, (double)x.y, s);
                s = fma((double)x.z, (double)x.z, s);
                s = fma((double)x.w, (double)x.w, s);
            }
        } else {
            for (int c = lane; c < d; c += 32) {
                const double x = acc[base + c];
                s = fma(x, x, s);
            }
        }
    }
    s = warp_sum_d(s);
    if (lane == 0) partials[w] = s;
}

// Pass 1 from per-row squared norms (4 bytes per touched row instead of the row itself).
__global__ void __launch_bounds__(256) touched_rowsq_kernel(const float* sqnorm, const int32_t* list,
                                                            const int32_t* count, double* partials) {
    const int lane = lane_id();
    const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= PARTIALS) return;
    const int n = *count;
    double s = 0.0;
    for (int i = w * 32 + lane; i < n; i += PARTIALS * 32) s += (double)sqnorm[list[i]];
    s = warp_sum_d(s);
    if (lane == 0) partials[w] = s;
}

// acc rows whose touched byte is 0 <- 0 (turns "untouched rows count as zero" into actual zeros).
__global__ void __launch_bounds__(256) zero_untouched_kernel(float* acc, const uint8_t* touched, int64_t rows, int d) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        if (touched[r]) continue;
        float* row = acc + r * d;
        for (int c = lane; c < d; c += 32) row[c] = 0.f;
    }
}

__global__ void norm_finish_kernel(const double* partials, float* out) {
    const int lane = lane_id();
    double s = 0.0;
    for (int i = lane; i < PARTIALS; i += 32) s += partials[i];
    s = warp_sum_d(s);
    if (lane == 0) *out = (float)sqrt(s);
}

}  // namespace smlm

using namespace smlm;

extern "C" size_t smlm_touched_workspace(int64_t rows) {
    TouchedBufs b;
    return layout_touched(std::max<int64_t>(rows, 0), nullptr, &b);
}

static int lazy_adam_impl(float* param, float* exp_avg, float* exp_avg_sq, float* acc, uint8_t* touched,
                          const float* grad_scale_dev, float grad_scale, int64_t rows, int64_t d, float one_minus_b1,
                          float b2, float one_minus_b2, float bc2_sqrt, float eps, float neg_step_size,
                          const float* scalars_dev, void* value_copy, int copy_dtype, int flags, void* workspace,
                          size_t workspace_bytes, void* stream) {
    SMLM_CHECK_ARG(rows >= 0 && d >= 0, "lazy_adam_step: negative size");
    SMLM_CHECK_ARG(rows < (int64_t)0x7fffffff, "lazy_adam_step: rows must be below 2^31");
    SMLM_CHECK_ARG(d < (1 << 30), "lazy_adam_step: d too large");
    SMLM_CHECK_ARG(value_copy == nullptr || copy_dtype == SMLM_F32 || copy_dtype == SMLM_BF16,
                   "lazy_adam_step: value copy must be fp32 or bf16");
    SMLM_CHECK_ARG((flags & ~SMLM_STEP_KEEP_ACC) == 0, "lazy_adam_step: unknown flags %d", flags);
    if (rows == 0) return SMLM_OK;
    SMLM_CHECK_ARG(param && exp_avg && exp_avg_sq && acc && touched, "lazy_adam_step: null pointer");
    cudaStream_t st = as_stream(stream);
    TouchedBufs b;
    int rc = compact_touched(touched, rows, workspace, workspace_bytes, &b, st);
    if (rc != SMLM_OK) return rc;
    AdamArgs a{param, exp_avg, exp_avg_sq, acc, touched, b.list, b.count, grad_scale_dev, grad_scale, (int)d,
               one_minus_b1, b2, one_minus_b2, bc2_sqrt, eps, neg_step_size, value_copy, copy_dtype,
               (flags & SMLM_STEP_KEEP_ACC) ? 1 : 0, scalars_dev};
    const bool vec = d % 4 == 0 && reinterpret_cast<uintptr_t>(param) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(exp_avg) % 16 == 0 && reinterpret_cast<uintptr_t>(exp_avg_sq) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(acc) % 16 == 0 &&
                     (value_copy == nullptr || reinterpret_cast<uintptr_t>(value_copy) % 16 == 0);
    const int blocks = persistent_blocks(8, 8);
    if (vec) lazy_adam_kernel<4><<<blocks, 256, 0, st>>>(a);
    else lazy_adam_kernel<1><<<blocks, 256, 0, st>>>(a);
    SMLM_LAUNCHED("lazy_adam_kernel");
    return SMLM_OK;
}

extern "C" int smlm_lazy_adam_step(float* param, float* exp_avg, float* exp_avg_sq, float* acc, uint8_t* touched,
                                   const float* grad_scale_dev, float grad_scale, int64_t rows, int64_t d,
                                   float one_minus_b1, float b2, float one_minus_b2, float bc2_sqrt, float eps,
                                   float neg_step_size, void* value_copy, int copy_dtype, int flags, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    return lazy_adam_impl(param, exp_avg, exp_avg_sq, acc, touched, grad_scale_dev, grad_scale, rows, d, one_minus_b1,
                          b2, one_minus_b2, bc2_sqrt, eps, neg_step_size, nullptr, value_copy, copy_dtype, flags,
                          workspace, workspace_bytes, stream);
}

extern "C" int smlm_lazy_adam_step_dev(float* param, float* exp_avg, float* exp_avg_sq, float* acc, uint8_t* touched,
                                       const float* grad_scale_dev, float grad_scale, int64_t rows, int64_t d,
                                       const float* scalars_dev, void* value_copy, int copy_dtype, int flags,
                                       void* workspace, size_t workspace_bytes, void* stream) {
    SMLM_CHECK_ARG(scalars_dev != nullptr, "lazy_adam_step_dev: null scalars");
    return lazy_adam_impl(param, exp_avg, exp_avg_sq, acc, touched, grad_scale_dev, grad_scale, rows, d, 0.f, 0.f,
                          0.f, 0.f, 0.f, 0.f, scalars_dev, value_copy, copy_dtype, flags, workspace, workspace_bytes,
                          stream);
}

extern "C" int smlm_lazy_adam_lowmem_step(float* param, void* exp_avg, void* exp_avg_sq, float* exp_avg_scale,
                                          float* exp_avg_sq_scale, int state_dtype, float* acc, uint8_t* touched,
                                          const float* grad_scale_dev, float grad_scale, int64_t rows, int64_t d,
                                          float beta1, float beta2, float one_minus_b1, float one_minus_b2, float eps,
                                          float step_size, float bc2_sqrt, void* value_copy, int copy_dtype,
                                          int flags, void* workspace, size_t workspace_bytes, void* stream) {
    SMLM_CHECK_ARG(rows >= 0 && d > 0, "lazy_adam_lowmem_step: rows must be >= 0 and the width > 0");
    SMLM_CHECK_ARG(rows < (int64_t)0x7fffffff && d < (1 << 30), "lazy_adam_lowmem_step: size too large");
    SMLM_CHECK_ARG(state_dtype == SMLM_BF16 || state_dtype == SMLM_I8,
                   "lazy_adam_lowmem_step: state must be bf16 or int8 (SMLM_BF16 / SMLM_I8)");
    SMLM_CHECK_ARG(value_copy == nullptr || copy_dtype == SMLM_F32 || copy_dtype == SMLM_BF16,
                   "lazy_adam_lowmem_step: value copy must be fp32 or bf16");
    SMLM_CHECK_ARG((flags & ~SMLM_STEP_KEEP_ACC) == 0, "lazy_adam_lowmem_step: unknown flags %d", flags);
    if (rows == 0) return SMLM_OK;
    SMLM_CHECK_ARG(param && exp_avg && exp_avg_sq && acc && touched, "lazy_adam_lowmem_step: null pointer");
    SMLM_CHECK_ARG(state_dtype != SMLM_I8 || (exp_avg_scale && exp_avg_sq_scale),
                   "lazy_adam_lowmem_step: int8 state needs both row scales");
    cudaStream_t st = as_stream(stream);
    TouchedBufs b;
    int rc = compact_touched(touched, rows, workspace, workspace_bytes, &b, st);
    if (rc != SMLM_OK) return rc;
    LowArgs a{param, acc, exp_avg, exp_avg_sq, exp_avg_scale, exp_avg_sq_scale, touched, b.list, b.count,
              grad_scale_dev, grad_scale, (int)d, beta1, beta2, one_minus_b1, one_minus_b2, eps, step_size,
              bc2_sqrt, value_copy, copy_dtype, (flags & SMLM_STEP_KEEP_ACC) ? 1 : 0};
    const int blocks = persistent_blocks(8, 8);
    const bool i8 = state_dtype == SMLM_I8;
    auto go = [&](auto NSc) {
        constexpr int NS = decltype(NSc)::value;
        if (i8) lazy_adam_lowmem_kernel<true, NS><<<blocks, 256, 0, st>>>(a);
        else lazy_adam_lowmem_kernel<false, NS><<<blocks, 256, 0, st>>>(a);
    };
    if (d <= 32 * 4) go(std::integral_constant<int, 4>{});
    else if (d <= 32 * 12) go(std::integral_constant<int, 12>{});
    else if (d <= 32 * 16) go(std::integral_constant<int, 16>{});
    else go(std::integral_constant<int, 0>{});
    SMLM_LAUNCHED("lazy_adam_lowmem_kernel");
    return SMLM_OK;
}

extern "C" int smlm_rowwise_step(float* param, float* acc, uint8_t* touched, float* v, int32_t* count,
                                 const float* grad_scale_dev, float grad_scale, int64_t rows, int64_t d, int kind,
                                 float b2, float eps, float lr, int flags, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    SMLM_CHECK_ARG(rows >= 0 && d > 0, "rowwise_step: rows must be >= 0 and the width > 0");
    SMLM_CHECK_ARG(rows < (int64_t)0x7fffffff && d < (1 << 30), "rowwise_step: size too large");
    SMLM_CHECK_ARG(kind == SMLM_ROWRMS || kind == SMLM_ROWADAGRAD, "rowwise_step: unknown kind %d", kind);
    SMLM_CHECK_ARG(kind != SMLM_ROWRMS || count != nullptr, "rowwise_step: rowrms needs the per-row count");
    SMLM_CHECK_ARG((flags & ~SMLM_STEP_KEEP_ACC) == 0, "rowwise_step: unknown flags %d", flags);
    if (rows == 0) return SMLM_OK;
    SMLM_CHECK_ARG(param && acc && touched && v, "rowwise_step: null pointer");
    cudaStream_t st = as_stream(stream);
    TouchedBufs b;
    int rc = compact_touched(touched, rows, workspace, workspace_bytes, &b, st);
    if (rc != SMLM_OK) return rc;
    RowArgs a{param,      acc,         v,     count, touched, b.list, b.count, grad_scale_dev, grad_scale, (int)d,
              kind,       b2,          eps,   lr,    (flags & SMLM_STEP_KEEP_ACC) ? 1 : 0};
    const int blocks = persistent_blocks(8, 8);
    const bool vec = d % 4 == 0 && reinterpret_cast<uintptr_t>(param) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(acc) % 16 == 0;
    switch (vec ? rowwise_groups(d) : -1) {
        case 1: rowwise_kernel<4, 1><<<blocks, 256, 0, st>>>(a); break;
        case 2: rowwise_kernel<4, 2><<<blocks, 256, 0, st>>>(a); break;
        case 3: rowwise_kernel<4, 3><<<blocks, 256, 0, st>>>(a); break;
        case 4: rowwise_kernel<4, 4><<<blocks, 256, 0, st>>>(a); break;
        case 0: rowwise_kernel<4, 0><<<blocks, 256, 0, st>>>(a); break;
        default: rowwise_kernel<1, 0><<<blocks, 256, 0, st>>>(a); break;
    }
    SMLM_LAUNCHED("rowwise_kernel");
    return SMLM_OK;
}

extern "C" int smlm_touched_norm(const float* acc, const float* row_sqnorm, const uint8_t* touched, int64_t rows,
                                 int64_t d, float* norm_out, void* workspace, size_t workspace_bytes, void* stream) {
    SMLM_CHECK_ARG(rows >= 0 && d >= 0, "touched_norm: negative size");
    SMLM_CHECK_ARG(rows < (int64_t)0x7fffffff && d < (1 << 30), "touched_norm: size too large");
    SMLM_CHECK_ARG(norm_out != nullptr, "touched_norm: null output");
    cudaStream_t st = as_stream(stream);
    if (rows == 0 || d == 0) {
        SMLM_CUDA(cudaMemsetAsync(norm_out, 0, sizeof(float), st));
        return SMLM_OK;
    }
    SMLM_CHECK_ARG((acc || row_sqnorm) && touched, "touched_norm: null pointer");
    TouchedBufs b;
    int rc = compact_touched(touched, rows, workspace, workspace_bytes, &b, st);
    if (rc != SMLM_OK) return rc;
    if (row_sqnorm)
        touched_rowsq_kernel<<<PARTIALS / 8, 256, 0, st>>>(row_sqnorm, b.list, b.count, b.partials);
    else if (d % 4 == 0 && reinterpret_cast<uintptr_t>(acc) % 16 == 0)
        touched_sq_kernel<4><<<PARTIALS / 8, 256, 0, st>>>(acc, b.list, b.count, (int)d, b.partials);
    else
        touched_sq_kernel<1><<<PARTIALS / 8, 256, 0, st>>>(acc, b.list, b.count, (int)d, b.partials);
    SMLM_LAUNCHED("touched_sq_kernel");
    norm_finish_kernel<<<1, 32, 0, st>>>(b.partials, norm_out);
    SMLM_LAUNCHED("norm_finish_kernel");
    return SMLM_OK;
}

extern "C" int smlm_zero_untouched(float* acc, const uint8_t* touched, int64_t rows, int64_t d, void* stream) {
    SMLM_CHECK_ARG(rows >= 0 && d >= 0 && d < (1 << 30), "zero_untouched: bad sizes");
    if (rows == 0 || d == 0) return SMLM_OK;
    SMLM_CHECK_ARG(acc && touched, "zero_untouched: null pointer");
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 16));
    zero_untouched_kernel<<<blocks, 256, 0, as_stream(stream)>>>(acc, touched, rows, (int)d);
    SMLM_LAUNCHED("zero_untouched_kernel");
    return SMLM_OK;
}
