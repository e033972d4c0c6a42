// Value tables in host RAM (the reference's host_values.py / host_rows.c path, re-designed for a GPU that can
// read and write host memory directly): the table, its gradient accumulator and its optimizer state stay in host
// RAM, page-locked and mapped into the device's address space (cudaHostRegister); the library's kernels then work
// on the rows a step reads straight over the host link (zero-copy, 16-byte accesses), with no CPU loop and no
// staging copy through the CPU:
//   * smlm_host_rows_gather: the distinct rows a forward reads, from the mapped table (or, for HOT rows and rows the
//     previous step updated, from their device copies) into a device tensor that the bag kernels then read;
//   * smlm_host_rows_scatter: rows updated on the device written back into the mapped table (the write-back of a
//     GACC step, which may run on another stream while the next step reads other rows);
//   * smlm_host_rows_add: a backward's per-row gradient sums (device) added into the mapped accumulator rows,
//     touched marks set, and the rows' squared norms kept on the device for the clip norm;
//   * smlm_rows_rowwise_step: the row-wise optimizer (rowrms / rowadagrad) over a list of rows with their gradients
//     in a device tensor (GACC: the step's gradient sums kept on the GPU) and, optionally, their current values in
//     another (the rows the forward gathered), table and state anywhere mapped: the table is then only written.
// The per-row optimizer steps over the mapped accumulator reuse smlm_lazy_adam_step, smlm_lazy_adam_lowmem_step and
// smlm_rowwise_step unchanged (their pointers may be mapped host memory).
#include "common.cuh"

namespace smlm {

// out[i] = slot[i] >= 0 ? hot[slot[i]] : slot2[i] >= 0 ? cache[slot2[i]] : table[rows[i]] (rows of d values,
// float4 lanes; one warp per row; slot / slot2 may be NULL).
__global__ void __launch_bounds__(256) host_gather_kernel(const float* table, const int64_t* rows,
                                                          const int32_t* slot, const float* hot, const int32_t* slot2,
                                                          const float* cache, int64_t n, int64_t table_rows, int d,
                                                          float* out, int* status) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int32_t s = slot ? slot[i] : -1;
        const int32_t s2 = slot2 ? slot2[i] : -1;
        const int64_t r = rows[i];
        const float* src;
        if (s >= 0) {
            src = hot + (int64_t)s * d;
        } else if (s2 >= 0) {
            src = cache + (int64_t)s2 * d;
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

// table[rows[i]] = values[i] (rows distinct; one warp per row, float4 lanes): the write-back of rows updated on the
// device into a mapped host table.
__global__ void __launch_bounds__(256) host_scatter_kernel(float* table, const int64_t* rows, const float* values,
                                                           int64_t n, int64_t table_rows, int d, int* status) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int64_t r = rows[i];
        if (r < 0 || r >= table_rows) {
            if (lane == 0) flag(status, SMLM_FLAG_INDEX_RANGE);
            continue;
        }
        const float* src = values + i * d;
        float* dst = table + r * d;
        for (int c = lane * 4; c < d; c += 128)
            *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
    }
}

// acc[rows[i]] = acc[rows[i]] + grads[i], touched[rows[i]] = 1, for the rows with skip[i] < 0 (rows distinct); a row
// whose touched mark is 0 gets 0 + grads[i] without its old value being read (the optimizer steps leave stepped
// rows' accumulators as they are, so a step's first add writes them: one crossing of the host link instead of
// three); with row_sq, also row_sq[rows[i]] = the new row's squared L2 norm (summed in double, stored fp32), so the
// clip norm needs no second pass over the accumulator rows.
__global__ void __launch_bounds__(256) host_add_kernel(float* acc, uint8_t* touched, float* row_sq, const int64_t* rows,
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
        const bool fresh = touched != nullptr && touched[r] == 0;
        double sq = 0.0;
        for (int c = lane * 4; c < d; c += 128) {
            float4 a = fresh ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<float4*>(dst + c);
            const float4 g = *reinterpret_cast<const float4*>(src + c);
            a.x = a.x + g.x; a.y = a.y + g.y; a.z = a.z + g.z; a.w = a.w + g.w;
            *reinterpret_cast<float4*>(dst + c) = a;
            sq = fma((double)a.x, (double)a.x, sq);
            sq = fma((double)a.y, (double)a.y, sq);
            sq = fma((double)a.z, (double)a.z, sq);
            sq = fma((double)a.w, (double)a.w, sq);
        }
        if (row_sq) {
            sq = warp_sum_d(sq);
            if (lane == 0) row_sq[r] = (float)sq;
        }
        __syncwarp();                      // every lane has read the mark before lane 0 sets it
        if (lane == 0 && touched) touched[r] = 1;
    }
}

// The row-wise step of rows[i] with gradient grads[i] (a device tensor of the step's row sums): rowwise_kernel's
// arithmetic in rowwise_kernel's order (rowwise_row), one warp per row; rows distinct. The row's current values
// come from current[i] when given (the copy the forward gathered onto the device, so the table is only written)
// and from the table otherwise; with to_current the updated row goes back into current[i] and the table is not
// touched (its write-back is a separate smlm_host_rows_scatter).
template <int VEC, int NC>
__global__ void __launch_bounds__(256) rows_rowwise_kernel(float* p, const int64_t* rows, const float* grads,
                                                           float* current, int64_t n, int64_t table_rows, int d,
                                                           float* row_v, int32_t* row_count, int kind, float b2,
                                                           float eps, float lr, const float* scale_dev, float scale,
                                                           int to_current, int* status) {
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const float sc = scale_dev ? *scale_dev : scale;
    for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
        const int64_t r = rows[i];
        if (r < 0 || r >= table_rows) {
            if (lane == 0) flag(status, SMLM_FLAG_INDEX_RANGE);
            continue;
        }
        float* pr = to_current ? current + i * d : p + r * d;
        rowwise_row<VEC, NC>(grads + i * d, false, current ? current + i * d : pr, pr, d, sc, kind, b2, eps, lr, row_v,
                             row_count, r, lane);
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

static bool aligned16(const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; }

extern "C" int smlm_host_rows_gather(const float* table, int64_t table_rows, const int64_t* rows, const int32_t* slot,
                                     const float* hot, const int32_t* slot2, const float* cache, int64_t n, int64_t d,
                                     float* out, int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && table_rows >= 0 && d > 0 && d % 4 == 0, "host_rows_gather: bad sizes (d %% 4 == 0)");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(table && rows && out && (slot == nullptr || hot != nullptr) && (slot2 == nullptr || cache != nullptr),
                   "host_rows_gather: null pointer");
    SMLM_CHECK_ARG(aligned16(table) && aligned16(out) && aligned16(hot) && aligned16(cache),
                   "host_rows_gather: table, hot, cache and out must be 16-byte aligned");
    host_gather_kernel<<<host_rows_blocks(n), 256, 0, as_stream(stream)>>>(table, rows, slot, hot, slot2, cache, n,
                                                                          table_rows, (int)d, out, status);
    SMLM_LAUNCHED("host_gather_kernel");
    return SMLM_OK;
}

extern "C" int smlm_host_rows_scatter(float* table, int64_t table_rows, const int64_t* rows, const float* values,
                                      int64_t n, int64_t d, int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && table_rows >= 0 && d > 0 && d % 4 == 0, "host_rows_scatter: bad sizes (d %% 4 == 0)");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(table && rows && values, "host_rows_scatter: null pointer");
    SMLM_CHECK_ARG(aligned16(table) && aligned16(values), "host_rows_scatter: table and values must be 16-byte aligned");
    // A quarter of the SMs, one block each: the copy is bound by the host link, which ~300 warps keep full, and a
    // write-back running beside the next step's kernels must leave them the other SMs. Its blocks ask for the
    // largest shared-memory carveout (they use none), so a kernel with a large shared-memory footprint can still
    // be placed beside them on the same SM.
    static bool carveout = false;
    if (!carveout) {
        SMLM_CUDA(cudaFuncSetAttribute(host_scatter_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       (int)cudaSharedmemCarveoutMaxShared));
        carveout = true;
    }
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, std::max(1, sm_count() / 4)));
    host_scatter_kernel<<<blocks, 256, 0, as_stream(stream)>>>(table, rows, values, n, table_rows, (int)d, status);
    SMLM_LAUNCHED("host_scatter_kernel");
    return SMLM_OK;
}

extern "C" int smlm_host_rows_add(float* acc, uint8_t* touched, float* row_sqnorm, int64_t table_rows,
                                  const int64_t* rows, const float* grads, const int32_t* skip, int64_t n, int64_t d,
                                  int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && table_rows >= 0 && d > 0 && d % 4 == 0, "host_rows_add: bad sizes (d %% 4 == 0)");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG(acc && rows && grads, "host_rows_add: null pointer");
    SMLM_CHECK_ARG(reinterpret_cast<uintptr_t>(acc) % 16 == 0 && reinterpret_cast<uintptr_t>(grads) % 16 == 0,
                   "host_rows_add: acc and grads must be 16-byte aligned");
    host_add_kernel<<<host_rows_blocks(n), 256, 0, as_stream(stream)>>>(acc, touched, row_sqnorm, rows, grads, skip, n,
                                                                       table_rows, (int)d, status);
    SMLM_LAUNCHED("host_add_kernel");
    return SMLM_OK;
}

extern "C" int smlm_rows_rowwise_step(float* param, int64_t table_rows, const int64_t* rows, const float* grads,
                                      float* current, int64_t n, int64_t d, float* row_v, int32_t* row_count,
                                      int kind, float beta2, float eps, float lr, const float* grad_scale_dev,
                                      float grad_scale, int flags, int* status, void* stream) {
    SMLM_CHECK_ARG(n >= 0 && table_rows >= 0 && d > 0, "rows_rowwise_step: bad sizes");
    SMLM_CHECK_ARG(kind == SMLM_ROWRMS || kind == SMLM_ROWADAGRAD, "rows_rowwise_step: unknown kind %d", kind);
    SMLM_CHECK_ARG(kind != SMLM_ROWRMS || row_count != nullptr, "rows_rowwise_step: rowrms needs the row counts");
    SMLM_CHECK_ARG((flags & ~SMLM_ROWS_TO_CURRENT) == 0, "rows_rowwise_step: unknown flags %d", flags);
    const int to_current = (flags & SMLM_ROWS_TO_CURRENT) ? 1 : 0;
    SMLM_CHECK_ARG(!to_current || current != nullptr, "rows_rowwise_step: SMLM_ROWS_TO_CURRENT needs current");
    if (n == 0) return SMLM_OK;
    SMLM_CHECK_ARG((param || to_current) && rows && grads && row_v, "rows_rowwise_step: null pointer");
    const bool vec = d % 4 == 0 && aligned16(param) && aligned16(grads) && aligned16(current);
    const int blocks = host_rows_blocks(n);
    cudaStream_t st = as_stream(stream);
#define SMLM_ROWS_ROWWISE(V, G)                                                                                    \
    rows_rowwise_kernel<V, G><<<blocks, 256, 0, st>>>(param, rows, grads, current, n, table_rows, (int)d, row_v,     \
                                                     row_count, kind, beta2, eps, lr, grad_scale_dev, grad_scale,  \
                                                     to_current, status)
    switch (vec ? rowwise_groups(d) : -1) {
        case 1: SMLM_ROWS_ROWWISE(4, 1); break;
        case 2: SMLM_ROWS_ROWWISE(4, 2); break;
        case 3: SMLM_ROWS_ROWWISE(4, 3); break;
        case 4: SMLM_ROWS_ROWWISE(4, 4); break;
        case 0: SMLM_ROWS_ROWWISE(4, 0); break;
        default: SMLM_ROWS_ROWWISE(1, 0); break;
    }
#undef SMLM_ROWS_ROWWISE
    SMLM_LAUNCHED("rows_rowwise_kernel");
    return SMLM_OK;
}
