"""oscar_b200 -- B200-native OSCAR INT2 rotated KV-cache hot path.

Package layout:
  plugin.py     vllm.general_plugins entry point and impl class surgery
  backend.py    OSCAR attention impl (forward / do_kv_cache_update / staging)
  kernels.py    torch-facing kernel API over the C ABI (include/oscar_b200.h)
  _native.py    ctypes binding of the in-tree _lib/liboscar_b200.so
  csrc/         sm_100a CUDA kernels and the C ABI
  format.py     INT2 slot layout constants
  config.py     OSCAR_ASCEND_* configuration
  rotation.py   per-layer rotation checkpoints
  mtp_shadow.py MTP draft-layer bf16 shadow pool
  synthetic.py  seeded synthetic workloads (tests, bench)
"""
from . import config, format, rotation  # noqa: F401

__version__ = "0.1.0"
__all__ = ["config", "format", "rotation", "__version__"]
