"""fsctep_b200 -- B200-native (sm_100a) rebuild of FSCTEP's per-edge Cartesian tensor-product
message-passing path (pure-cartesian-ictd, pure-cartesian-ictd-o3 and pure-cartesian-sparse) and
its force/virial backward.

Compute lives in ``_lib/libfsctep_b200.so`` (CUDA C++ behind the C ABI of
``include/fsctep_b200.h``); this package is the host-side mirror of the reference's
operator surface.  There is no CPU fallback.
"""

__version__ = "0.1.0"
