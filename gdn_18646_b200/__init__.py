"""gdn_18646_b200 -- B200 (sm_100a) Gated DeltaNet hot path.

The compute lives in ``lib/libgdn_b200.so`` (C ABI: ``include/gdn_b200.h``);
this package is the torch-facing host side: the functional ops and the
reference-surface ``exts()`` modules.
"""
from . import _lib
from .ops import (CHUNK, DecodeModule, PrefillModule, ProjModule, RMSNormModule, decode_proj, decode_step, exts,
                  gated_rmsnorm, prefill, prefill_varlen, proj_conv_silu, rmsnorm)

__all__ = ["CHUNK", "DecodeModule", "PrefillModule", "ProjModule", "RMSNormModule", "decode_proj", "decode_step", "exts",
           "gated_rmsnorm", "prefill", "prefill_varlen", "proj_conv_silu", "rmsnorm", "_lib"]
