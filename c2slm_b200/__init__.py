"""c2slm_b200: the token loop of hazyhaar/c2slm (engine.Forward -> ComputeLogits
-> repetition penalty -> greedy argmax) as sm_100a CUDA behind a C ABI
(include/c2slm_b200.h), with a Python host mirror of the reference API."""
from .engine import (C2SError, Engine, F32, Q4_K, Q5_0, Q6_K, Q8_0, dequant_row, dot_rows_f32x,  # noqa: F401
                     gemv, kquant_partials, load_library, quantize_row_q8_k, rmsnorm, swiglu)

__version__ = "0.1.0"
