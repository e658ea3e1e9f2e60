"""B200-native (sm_100a) Local Token Hyper-Connection interface.

The kernels live in ``liblthc_b200.so`` (C ABI, ``include/lthc_b200.h``).
``ops`` exposes them as PyTorch operators with autograd; ``modules`` mirrors the
reference's ``SharedLocalRead`` / ``LayerLocalWrite`` modules; ``integration``
installs the kernels behind an existing ``flowmatching_lthc`` model.
"""
from . import _lib, ops  # noqa: F401
from .ops import (  # noqa: F401
    final_accumulate_b4_12_traceable,
    lazy_update,
    materialise,
    read,
    weight_grad,
    write,
    write_add,
)

__version__ = "0.1.0"
