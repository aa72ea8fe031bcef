"""B200-native VC-attention library: C-ABI CUDA kernels for sm_100a
(``libvc_b200.so``) and thin torch wrappers (``vc_b200.ops``)."""
from . import ops  # noqa: F401
