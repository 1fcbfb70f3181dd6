"""B200-native (sm_100a) Spark-H3 adaptive block-sparse attention."""
from . import ops
from .ops import spark_layer

__all__ = ["ops", "spark_layer"]
