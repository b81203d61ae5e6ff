"""spark_b200: B200-native (sm_100a) decode hot path of Spark-MLX-LLM.

* ``spark_b200.ops``      - ``torch.ops.spark_b200.*`` custom operators.
* ``spark_b200.ext``      - the ``spark_mlx_ext`` function signatures.
* ``spark_b200.dispatch`` - the ``spark_mlx_llm.ops`` dispatch layer.
* ``spark_b200.decoder``  - the synthetic 4B-class decoder (1 GPU or TP).

All compute runs in ``lib/libsparkb200.so`` (C ABI in include/spark_b200.h);
importing an operator without the library raises ``RuntimeError``.
"""

from . import dispatch, ext, ops  # noqa: F401  (ops registers torch.ops.spark_b200.*)
from ._lib import LIB_PATH, lib  # noqa: F401

__version__ = "0.1.0"
