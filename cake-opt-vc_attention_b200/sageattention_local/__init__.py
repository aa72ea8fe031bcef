"""B200 (sm_100a) drop-in for the reference ``sageattention_local`` VC entry
points: ``sageattn_vc`` plus the private ``prepare`` / ``forward_prepared``
split, ``sage_vc_build_info`` and ``kernel_resources``."""
from .vc import (forward_prepared, kernel_resources, prepare, sage_vc_build_info, sageattn_vc,  # noqa: F401
                 validate_inputs)

__all__ = ["sageattn_vc", "prepare", "forward_prepared", "sage_vc_build_info", "kernel_resources",
           "validate_inputs"]
