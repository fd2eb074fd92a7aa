"""SiliconGraph-B200: the quantized transformer-block path of SiliconGraph
(weight-only INT4/INT8 linear + causal flash attention) as hand-written
sm_100a CUDA behind a C ABI (include/sg_kernels.h, include/armcc_sdk.h).

Python here is a thin host binding used by tests and the benchmark; the
kernels and the runtime are native (lib/libsg_b200.so)."""
from ._lib import LIB_PATH, SgError, load  # noqa: F401

__version__ = "0.1.0"
