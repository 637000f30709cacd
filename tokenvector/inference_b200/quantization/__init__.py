"""Mirror of the reference's tv.quantization package (engine, matmul, types, int4)."""
from .engine import *  # noqa: F401,F403
from .int4 import *  # noqa: F401,F403
from .matmul import *  # noqa: F401,F403
from .types import (FP8E4M3, QuantParams, fp8e4m3_from_float, identity,  # noqa: F401
                    native_fp8_e4m3_decode, native_fp8_e4m3_encode)
