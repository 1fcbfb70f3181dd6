"""Public Spark names (h3_sparse_attention/spark.py:1-39).

``spark_reblock`` is the landmark-tree-v2 block builder (64-token leaves, the permutation and
its inverse); ``spark_reweight(a, k, v)`` returns the query-conditioned weighted keys, weighted
values and log-mass correction ``(ak, av, lm)``; ``spark_block`` is the initial public name
of ``spark_reblock``.  All three are the same objects the package root exports.
"""
from .attention import spark_reweight
from .processor import install_h3_spark_attn
from .reblock import spark_reblock

spark_block = spark_reblock

__all__ = ["spark_reblock", "spark_reweight", "spark_block", "install_h3_spark_attn"]
