"""daisychain-infer_b200: DaisyChain-Infer's verified INT8 W8A8 path on B200.

The compute lives in libdcinfer.so (hand-written CUDA for sm_100a behind the C
ABI of include/dcinfer.h).  This package is the host-side mirror of the
reference's compute-core interface (public/webgpu.js's compute object,
public/verified_core.js's contract, public/infer.js's stage API).
"""
from ._lib import AccumulatorBoundError, DeviceError, NonFiniteError  # noqa: F401
from .compute import Compute, Weight, init_compute  # noqa: F401
from . import infer, shard  # noqa: E402,F401
from . import pipeline  # noqa: E402,F401
from . import wire  # noqa: E402,F401
from . import safetensors  # noqa: E402,F401
