"""B200-native (sm_100a) Spark-H3 adaptive block-sparse attention.

Drop-in names of the reference package (`h3_sparse_attention`): the installers and config,
the attention seam `spark_attention_bthd`, and the standalone primitives `spark_reblock`
(alias `spark_block`) and `spark_reweight` (h3_sparse_attention/__init__.py:12-36).  Kernels live
in libsparkh3b200.so (C ABI, include/spark_h3_b200.h) and always run on the GPU.
"""
from .attention import spark_attention_bthd, spark_reweight
from .fp8_linear import Fp8Linear, convert_linear_to_fp8, install_fp8
from .config import H3SparseAttentionConfig
from .layout import PackedLayout, packed_layout
from .processor import (H3SparseAttentionPlugin, install_h3_sol_attn, install_h3_spark_attn,
                        install_h3_sparse_attention)
from .reblock import spark_reblock
from . import ops

spark_block = spark_reblock

__all__ = [
    "Fp8Linear", "H3SparseAttentionConfig", "H3SparseAttentionPlugin", "convert_linear_to_fp8", "install_fp8", "PackedLayout", "install_h3_spark_attn",
    "install_h3_sol_attn", "install_h3_sparse_attention", "ops", "packed_layout", "spark_attention_bthd",
    "spark_block", "spark_reblock", "spark_reweight",
]
