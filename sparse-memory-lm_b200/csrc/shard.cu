// Helpers of the row-sharded value table: ordered sum of the owners' partial results.
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

}  // namespace smlm

using namespace smlm;

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
