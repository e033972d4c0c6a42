"""B200 (sm_100a) product-key memory layer behind the API of re133/sparse-memory-lm's smlm package.

Modules mirror the reference's: kernels (the kernel layer, C ABI in include/smlm_b200.h), pkm
(ProductKeyMemory), sparse_values (RowStore, row-sparse bag, LazyRowAdam), row_optim (RowWiseOptimizer),
optim (routing / clipping), model (decoder hosting the layers).
"""
__version__ = "0.1.0"
