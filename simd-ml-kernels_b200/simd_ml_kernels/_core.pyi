"""Type stubs of simd_ml_kernels._core, the B200 build's extension module.

Names, parameter order and defaults follow the reference package's stubs for
the same functions (the decode-GEMV path); the keyword-only `out=` and
`stream=` are this build's additions. Array arguments are NumPy arrays (host
memory: synchronous, as in the reference) or objects with
`__cuda_array_interface__` such as torch CUDA tensors (device memory:
asynchronous on `stream`, a raw cudaStream_t as an integer).
"""

from typing import Any, Optional

import numpy as np
from numpy.typing import NDArray

class DTypeError(TypeError, RuntimeError):
    """An array argument has the wrong dtype."""

class ArgumentError(ValueError, RuntimeError):
    """An argument has the wrong shape, layout or value."""

def version() -> str:
    """Library version, e.g. '0.1.0 (sm_100a)'."""
    ...

def sgemm(
    A: Any,
    B: Any,
    C: Optional[Any] = None,
    alpha: float = 1.0,
    beta: float = 0.0,
    isa: str = "",
    *,
    trans_a: bool = False,
    trans_b: bool = False,
    stream: Optional[int] = None,
) -> NDArray[np.float32]:
    """C = alpha * A @ B.T + beta * C (float32) for the decode shape: trans_b=True,
    trans_a=False, at most 8 rows of A. Other shapes raise ArgumentError."""
    ...

def sgemm_f16(
    A: Any,
    B: Any,
    alpha: float = 1.0,
    beta: float = 0.0,
    C: Optional[Any] = None,
    *,
    trans_b: bool = False,
    stream: Optional[int] = None,
) -> NDArray[np.float32]:
    """float16 A [M, K], B [N, K] (trans_b=True, M <= 8); float32 accumulation and output."""
    ...

def sgemm_bf16(
    A: Any,
    B: Any,
    alpha: float = 1.0,
    beta: float = 0.0,
    C: Optional[Any] = None,
    *,
    trans_b: bool = False,
    stream: Optional[int] = None,
) -> NDArray[np.float32]:
    """bfloat16 A and B (uint16 bit patterns or ml_dtypes.bfloat16), trans_b=True,
    M <= 8; float32 accumulation and output."""
    ...

def sgemm_u8s8(
    A: Any,
    B: Any,
    a_scale: float,
    a_zero_point: int,
    b_scales: Any,
    C: Optional[Any] = None,
    *,
    trans_b: bool = False,
    stream: Optional[int] = None,
) -> NDArray[np.float32]:
    """C = a_scale * b_scales[j] * sum_k (A - a_zero_point) * B[j, k]: uint8 A [M, K]
    (M <= 8), int8 B [N, K] with trans_b=True; exact integer sums and the
    reference's scalar-table rounding."""
    ...

def quantize_q4_0(W: Any, *, out: Optional[Any] = None, stream: Optional[int] = None) -> NDArray[np.uint8]:
    """ggml Q4_0 blocks of W [..., K], K % 32 == 0: uint8 [..., K/32*18]."""
    ...

def quantize_q8_0(W: Any, *, out: Optional[Any] = None, stream: Optional[int] = None) -> NDArray[np.uint8]:
    """ggml Q8_0 blocks of W [..., K], K % 32 == 0: uint8 [..., K/32*34]."""
    ...

def gemv_q4_0(
    x: Any, Wq: Any, N: int, K: int, *, out: Optional[Any] = None, stream: Optional[int] = None
) -> NDArray[np.float32]:
    """y = x @ W.T [N] for x [K], W as N rows of Q4_0 blocks."""
    ...

def gemv_q8_0(
    x: Any, Wq: Any, N: int, K: int, *, out: Optional[Any] = None, stream: Optional[int] = None
) -> NDArray[np.float32]:
    """y = x @ W.T [N] for x [K], W as N rows of Q8_0 blocks."""
    ...

def gemv_q4_0_batch(
    x: Any, Wq: Any, N: int, K: int, *, out: Optional[Any] = None, stream: Optional[int] = None
) -> NDArray[np.float32]:
    """Y = X @ W.T [M, N] for up to 8 rows of X [M, K] (an addition of this build)."""
    ...

def gemv_q8_0_batch(
    x: Any, Wq: Any, N: int, K: int, *, out: Optional[Any] = None, stream: Optional[int] = None
) -> NDArray[np.float32]:
    """Y = X @ W.T [M, N] for up to 8 rows of X [M, K] (an addition of this build)."""
    ...

def gemv_dense(
    x: Any, W: Any, wtype: str = "float32", out: Optional[Any] = None, stream: Optional[int] = None
) -> NDArray[np.float32]:
    """Y = X @ W.T for float32 X [M, K] (M <= 8), W [N, K] in float32, float16 or
    bfloat16 (an addition of this build)."""
    ...
