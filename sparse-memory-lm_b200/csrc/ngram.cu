// Engram n-gram rows: the hash of the reference's NgramHash.forward (smlm/engram.py:63-75) in one pass.
//
// For position t of sequence b and lookup (order o, head h): x = XOR over i < orders[o] of
// c[b, history + t - i] * mult[o, h, i] (int64), x ^= x >> 17, row = x mod rows (floor) + (o * heads + h) * rows.
// One thread per (b, t, lookup); the lookups of a position are contiguous in the output, so a warp writes
// consecutive int64s. Integer arithmetic only: bit-identical to the reference's tensor expression.
#include "common.cuh"

namespace smlm {

constexpr int NGRAM_MAX_ORDERS = 8;

struct NgramArgs {
    const int64_t* c;
    const int64_t* mult;  // (n_orders, heads, max_order)
    int64_t* out;         // (batch, t_len, n_orders * heads)
    int64_t batch, t_len, rows;
    int history, n_orders, heads, max_order;
    int orders[NGRAM_MAX_ORDERS];
};

__global__ void __launch_bounds__(256) ngram_rows_kernel(NgramArgs a) {
    const int lookups = a.n_orders * a.heads;
    const int64_t total = a.batch * a.t_len * lookups;
    const int64_t width = a.history + a.t_len;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(i % lookups);
        const int64_t bt = i / lookups;
        const int64_t t = bt % a.t_len, b = bt / a.t_len;
        const int o = j / a.heads, h = j % a.heads;
        const int64_t* cb = a.c + b * width + a.history + t;
        const int64_t* m = a.mult + ((int64_t)o * a.heads + h) * a.max_order;
        int64_t x = 0;
        for (int k = 0; k < a.orders[o]; k++) x ^= __ldg(cb - k) * __ldg(m + k);
        x ^= x >> 17;
        int64_t r = x % a.rows;
        if (r < 0) r += a.rows;
        a.out[i] = r + (int64_t)j * a.rows;
    }
}

}  // namespace smlm

using namespace smlm;

extern "C" int smlm_ngram_rows(const int64_t* c, int64_t batch, int64_t t_len, int history, const int64_t* mult,
                               const int* orders, int n_orders, int heads, int max_order, int64_t rows, int64_t* out,
                               void* stream) {
    SMLM_CHECK_ARG(batch >= 0 && t_len >= 0 && history >= 0, "ngram_rows: negative size");
    SMLM_CHECK_ARG(n_orders >= 1 && n_orders <= NGRAM_MAX_ORDERS && heads >= 1 && max_order >= 1 && rows >= 1,
                   "ngram_rows: need 1 <= n_orders <= %d, heads >= 1, max_order >= 1, rows >= 1", NGRAM_MAX_ORDERS);
    SMLM_CHECK_ARG(orders != nullptr, "ngram_rows: null orders");
    NgramArgs a{c, mult, out, batch, t_len, rows, history, n_orders, heads, max_order, {}};
    for (int o = 0; o < n_orders; o++) {
        SMLM_CHECK_ARG(orders[o] >= 1 && orders[o] <= max_order && orders[o] <= history + 1,
                       "ngram_rows: order %d must be in [1, min(max_order, history + 1)]", orders[o]);
        a.orders[o] = orders[o];
    }
    const int64_t total = batch * t_len * n_orders * heads;
    if (total == 0) return SMLM_OK;
    SMLM_CHECK_ARG(c && mult && out, "ngram_rows: null pointer");
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 16));
    ngram_rows_kernel<<<blocks, 256, 0, as_stream(stream)>>>(a);
    SMLM_LAUNCHED("ngram_rows_kernel");
    return SMLM_OK;
}
