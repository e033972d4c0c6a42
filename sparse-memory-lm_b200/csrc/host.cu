// Value tables in host RAM (the reference's host_values.py / host_rows.c path, re-designed for a GPU that can
// read and write host memory directly): the table, its gradient accumulator and its optimizer state stay in host
// RAM, page-locked and mapped into the device's address space (cudaHostRegister); the library's kernels then work
// on the rows a step reads straight over the host link (zero-copy, 16-byte accesses), with no CPU loop and no
// staging copy through the CPU:
//   * smlm_host_rows_gather: the distinct rows a forward reads, from the mapped table (or, for HOT rows, from their
//     device copies) into a device tensor that the bag kernels then read;
//   * smlm_host_rows_add: a backward's per-row gradient sums (device) added into the mapped accumulator rows,
//     touched marks set;
//   * smlm_rows_rowwise_step: the row-wise optimizer (rowrms / rowadagrad) over a list of rows with their gradients
//     in a device tensor (GACC: the step's gradient sums kept on the GPU), table and state anywhere mapped.
// The per-row optimizer steps over the mapped accumulator reuse smlm_lazy_adam_step, smlm_lazy_adam_lowmem_step and
// smlm_rowwise_step unchanged (their pointers may be mapped host memory).
#include "common.cuh"

namespace smlm {

// out[i] = slot[i] >= 0 ? hot[slot[i]] : table[rows[i]] (rows of d values, float4 lanes; one warp per row).
__global__ void __launch_bounds__(256) host_gather_kernel(const float* table, const int64_t* rows,
                                                          const int32_t* slot, const float* hot, int64_t n,
                                                          int64_t table_rows, int d, float* out, int* status) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int32_t s = slot ? slot[i] : -1;
        const int64_t r = rows[i];
        const float* src;
        if (s >= 0) {
            src = hot + (int64_t)s * d;
        } else if (r >= 0 && r < table_rows) {
            src = table + r * d;
        } else {
            flag(status, SMLM_FLAG_INDEX_RANGE);
            src = nullptr;
        }
        float* dst = out + i * d;
        for (int c = lane * 4; c < d; c += 128) {
            const float4 v = src ? *reinterpret_cast<const float4*>(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(dst + c) = v;
        }
    }
}

// acc[rows[i]] = acc[rows[i]] + grads[i], touched[rows[i]] = 1, for the rows with skip[i] < 0 (rows distinct).
__global__ void __launch_bounds__(256) host_add_kernel(float* acc, uint8_t* touched, const int64_t* rows,
                                                       const float* grads, const int32_t* skip, int64_t n,
                                                       int64_t table_rows, int d, int* status) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        if (skip && skip[i] >= 0) continue;
        const int64_t r = rows[i];
        if (r < 0 || r >= table_rows) {
            if (lane == 0) flag(status, SMLM_FLAG_INDEX_RANGE);
            continue;
        }
        float* dst = acc + r * d;
        const float* src = grads + i * d;
        for (int c = lane * 4; c < d; c += 128) {
            float4 a = *reinterpret_cast<float4*>(dst + c);
            const float4 g = *reinterpret_cast<const float4*>(src + c);
            a.x = a.x + g.x; a.y = a.y + g.y; a.z = a.z + g.z; a.w = a.w + g.w;
            *reinterpret_cast<float4*>(dst + c) = a;
        }
        if (lane == 0 && touched) touched[r] = 1;
    }
}

// The row-wise step of rows[i] with gradient grads[i] (a device tensor of the step's row sums): rowwise_kernel's
// arithmetic in rowwise_kernel's order (q summed in double over each lane's VEC-column groups, then across the
// warp; rowwise_state_step; p -= step * g * scale), one warp per row; rows distinct.
template <int VEC>
__global__ void __launch_bounds__(256) rows_rowwise_kernel(float* p, const int64_t* rows, const float* grads,
                                                           int64_t n, int64_t table_rows, int d, float* row_v,
                                                           int32_t* row_count, int kind, float b2, float eps,
                                                           float lr, const float* scale_dev, float scale,
                                                           int* status) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const float sc = scale_dev ? *scale_dev : scale;
    for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int64_t r = rows[i];
        if (r < 0 || r >= table_rows) {
            if (lane == 0) flag(status, SMLM_FLAG_INDEX_RANGE);
            continue;
        }
        const float* g = grads + i * d;
        double q = 0.0;
        for (int c = lane * VEC; c < d; c += 32 * VEC) {
#pragma unroll
            for (int t = 0; t < VEC; t++) {
                const float gk = __fmul_rn(g[c + t], sc);
                q = fma((double)gk, (double)gk, q);
            }
        }
        q = warp_sum_d(q) / (double)d;
        const float step = rowwise_state_step(kind, b2, eps, lr, row_v, row_count, r, q, lane);
        float* pr = p + r * d;
        for (int c = lane * VEC; c < d; c += 32 * VEC) {
#pragma unroll
            for (int t = 0; t < VEC; t++)
                pr[c + t] = __fsub_rn(pr[c + t], __fmul_rn(step, __fmul_rn(g[c + t], sc)));
        }
    }
}

}  // namespace smlm

using namespace smlm;

extern "C" int smlm_host_register(void* ptr, size_t bytes, void** device_ptr) {
    SMLM_CHECK_ARG(ptr && bytes > 0 && device_ptr, "host_register: bad arguments");
    *device_ptr = nullptr;
    SMLM_CUDA(cudaHostRegister(ptr, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable));
    SMLM_CUDA(cudaHostGetDevicePointer(device_ptr, ptr, 0));
    return SMLM_OK;
}

extern "C" int smlm_host_unregister(void* ptr) {
    SMLM_CHECK_ARG(ptr, "host_unregister: null pointer");
    SMLM_CUDA(cudaHostUnregister(ptr));
    return SMLM_OK;
}

static int host_rows_blocks(int64_t n) {
    return (int)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, (int64_t)sm_count() * 16));
}

extern "C" int smlm_host_rows_gather(const float* table, int64_t table_rows, const int64_t* rows, const int32_t* slot,
                                     const float* hot, int64_t n, int64_t d, float* out, int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && table_rows >= 0 && d > 0 && d % 4 == 0, "host_rows_gather: bad sizes (d %% 4 == 0)");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(table && rows && out && (slot == nullptr || hot != nullptr), "host_rows_gather: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(table) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(hot) % 16 == 0,
                   "host_rows_gather: table, hot and out must be 16-byte aligned");
    host_gather_kernel<<<host_rows_blocks(n), 256, 0, as_stream(stream)>>>(table, rows, slot, hot, n, table_rows,
                                                                          (int)d, out, status);
    SMLM_LAUNCHED("host_gather_kernel");
    return SMLM_OK;
}

extern "C" int smlm_host_rows_add(float* acc, uint8_t* touched, int64_t table_rows, const int64_t* rows,
                                  const float* grads, const int32_t* skip, int64_t n, int64_t d, int* status,
                                  void* stream) {
    SMLM_CHECK_ARG(n >= 0 && table_rows >= 0 && d > 0 && d % 4 == 0, "host_rows_add: bad sizes (d %% 4 == 0)");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(acc && rows && grads, "host_rows_add: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(acc) % 16 == 0 && reinterpret_cast<uintptr_t>(grads) % 16 == 0,
                   "host_rows_add: acc and grads must be 16-byte aligned");
    host_add_kernel<<<host_rows_blocks(n), 256, 0, as_stream(stream)>>>(acc, touched, rows, grads, skip, n, table_rows,
                                                                       (int)d, status);
    SMLM_LAUNCHED("host_add_kernel");
    return SMLM_OK;
}

extern "C" int smlm_rows_rowwise_step(float* param, int64_t table_rows, const int64_t* rows, const float* grads,
                                      int64_t n, int64_t d, float* row_v, int32_t* row_count, int kind, float beta2,
                                      float eps, float lr, const float* grad_scale_dev, float grad_scale, int* status,
                                      void* stream) {
    SMLM_CHECK_ARG(n >= 0 && table_rows >= 0 && d > 0, "rows_rowwise_step: bad sizes");
    SMLM_CHECK_ARG(kind == SMLM_ROWRMS || kind == SMLM_ROWADAGRAD, "rows_rowwise_step: unknown kind %d", kind);
    SMLM_CHECK_ARG(kind != SMLM_ROWRMS || row_count != nullptr, "rows_rowwise_step: rowrms needs the row counts");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(param && rows && grads && row_v, "rows_rowwise_step: null pointer");
    if (d % 4 == 0)
        rows_rowwise_kernel<4><<<host_rows_blocks(n), 256, 0, as_stream(stream)>>>(
            param, rows, grads, n, table_rows, (int)d, row_v, row_count, kind, beta2, eps, lr, grad_scale_dev,
            grad_scale, status);
    else
        rows_rowwise_kernel<1><<<host_rows_blocks(n), 256, 0, as_stream(stream)>>>(
            param, rows, grads, n, table_rows, (int)d, row_v, row_count, kind, beta2, eps, lr, grad_scale_dev,
            grad_scale, status);
    SMLM_LAUNCHED("rows_rowwise_kernel");
    return SMLM_OK;
}
