"""B200-native GBDT training path of mojotrees (ajhendel/mojoboost).

Training runs in libmojotrees_b200.so (hand-written sm_100a CUDA behind the
reference's C ABI, include/mojotrees.h).  Python reaches it through ctypes;
there is no Python or CPU training fallback.
"""
from ._capi import (  # noqa: F401
    Model, MojoTreesError, UnsupportedError, abi_version, bin_dense, gpu_available, histogram_u8, lib,
    shared_atomic_peak, check_quotients, train_csc, bin_csc,
    nccl_unique_id, train_binned, train_binned_dp, train_dense,
)

__all__ = ["Model", "MojoTreesError", "UnsupportedError", "abi_version", "bin_dense",
           "check_quotients", "gpu_available", "histogram_u8", "lib", "nccl_unique_id", "shared_atomic_peak", "train_binned", "train_csc", "bin_csc",
           "train_binned_dp", "train_dense"]
