"""``quantaweave_b200.moe_kernels``: the reference's ``moe_kernels`` module name (``src/moe_kernels.py``), backed by the
tcgen05 grouped GEMM (see ``ops/grouped.py``)."""

from .ops.grouped import (GroupedPlan, benchmark, compute_dtype, experts_support_grouped, grouped_matmul,  # noqa: F401
                          grouped_swiglu, kernels_available)

__all__ = ["GroupedPlan", "benchmark", "compute_dtype", "experts_support_grouped", "grouped_matmul",
           "grouped_swiglu", "kernels_available"]
