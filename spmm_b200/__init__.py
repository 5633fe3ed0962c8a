"""spmm_b200 -- B200-native (sm_100a) SpMM for the BOO and PBR block-sparse formats.

A drop-in for the hot path of Dayan135/SPMM (``torch_fast_spdmm``): the same
Python API (``csr_to_boo`` / ``csr_to_pbr``, ``.to('cuda')``, ``boo_matmul`` /
``pbr_matmul`` and their helpers) over the C ABI in ``include/spmm_b200.h``,
implemented by hand-written CUDA for sm_100a in ``spmm_b200/csrc``.  Formats
are built on the GPU; every product runs on the GPU; there is no CPU fallback.
"""

from .boo import (BOOInfo, BOOMatrixInt32Double, BOOMatrixInt32Float, BOOMatrixInt64Double,
                  BOOMatrixInt64Float, BooNzOrder, BooSmallBlockPolicy, NZ_ORDERS,
                  SMALL_BLOCK_POLICIES, boo_arena_bytes, boo_info, boo_matmul, boo_to_csr,
                  check_product, csr_to_boo, product_status)
from .boo_plan import BOOExecutionPlan, prepare_boo_cuda
from .clustering import CLUSTER_METHODS, cluster_axes, cluster_axis
from .io import load_boo, load_pbr, save_boo, save_pbr
from .pbr import (BlockFillStats, BlockStripeStats, DataOrder, PBRInfo, PBRMatrixInt32Double,
                  PBRMatrixInt32Float, PBRMatrixInt64Double, PBRMatrixInt64Float, csr_to_pbr,
                  pbr_analyze_csr, pbr_batched_matmul_chunkcols_cuda, pbr_batched_matmul_cpu,
                  pbr_batched_matmul_cuda, pbr_batched_matmul_nnzflat_cuda,
                  pbr_batched_matmul_variant_cuda, pbr_info, pbr_matmul, pbr_to_csr)
from ._lib import SpmmError
from .timed import BOOTimedSpMM, DirectSpMM, PBRTimedSpMM

__all__ = [
    'csr_to_boo', 'boo_to_csr', 'boo_info', 'boo_matmul', 'boo_arena_bytes', 'BOOInfo',
    'product_status', 'check_product', 'SpmmError',
    'SMALL_BLOCK_POLICIES', 'NZ_ORDERS', 'cluster_axes', 'cluster_axis', 'CLUSTER_METHODS',
    'csr_to_pbr', 'pbr_to_csr', 'pbr_analyze_csr', 'pbr_info', 'PBRInfo', 'BlockFillStats',
    'BlockStripeStats', 'pbr_matmul', 'pbr_batched_matmul_cpu', 'pbr_batched_matmul_cuda',
    'pbr_batched_matmul_chunkcols_cuda', 'pbr_batched_matmul_nnzflat_cuda',
    'pbr_batched_matmul_variant_cuda', 'BOOExecutionPlan', 'prepare_boo_cuda',
    'BOOTimedSpMM', 'PBRTimedSpMM', 'DirectSpMM', 'save_boo', 'load_boo', 'save_pbr', 'load_pbr',
]
