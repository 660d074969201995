"""musapy_b200: musapy's stride-aware elementwise and reduction engine,
rebuilt for NVIDIA B200 (sm_100a).

``import musapy_b200 as ms`` gives the ``ms.*`` surface of musapy's hot path
(python/musapy/__init__.py:3-110): add/sub/mul/div/pow, sin/cos/exp/log/abs/
sign/neg, clamp, eq/ne/lt/gt/le/ge, sum/prod/max/min/mean/argmax/argmin/
cumsum, ``Array.astype`` and the dunders, plus the array creation and view
helpers those ops need. Every op runs on the CUDA kernels of
``_lib/libmusapy_b200.so``; there is no CPU execution path.
"""
from . import dtypes as _dtype_mod
from . import errors
from ._lib import LIB as _LIB
from .array import (
    Array,
    Device,
    array,
    broadcast_to,
    empty,
    flip,
    from_dlpack,
    from_numpy,
    from_torch,
    getitem,
    index_select,
    permute,
    reshape,
    set_default_device,
    set_default_dtype,
    slice,
    squeeze,
    transpose,
)
from .dtypes import (
    Dtype,
    bfloat16,
    bool_,
    complex64,
    complex128,
    float16,
    float32,
    float64,
    int8,
    int16,
    int32,
    int64,
    uint8,
    uint16,
    uint32,
    uint64,
)
from .streams import Stream, device, dtype, stream
from .errors import (
    DeviceError,
    DeviceNotConfiguredError,
    DtypeError,
    InteropError,
    KernelError,
    LinAlgError,
    MemoryError,
    MusapyError,
    OutOfMemoryError,
    ShapeError,
    StreamError,
)
from .ops import (
    abs,
    add,
    arange,
    argmax,
    argmin,
    astype,
    clamp,
    contiguous,
    cos,
    cumsum,
    div,
    eq,
    exp,
    eye,
    full,
    ge,
    gt,
    le,
    linspace,
    log,
    lt,
    max,
    mean,
    min,
    mul,
    ne,
    neg,
    ones,
    ones_like,
    pow,
    prod,
    sign,
    sin,
    sub,
    sum,
    zeros,
    zeros_like,
)

__version__ = "0.1.0"
bool = bool_  # noqa: A001 - musapy exports its bool dtype under this name


def library_path() -> str:
    from ._lib import LIB_PATH

    return LIB_PATH
