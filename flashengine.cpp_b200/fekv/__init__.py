"""fekv — host-side binding of the B200 paged-KV hot path.

* :mod:`fekv._lib`      ctypes binding of ``include/fe_kv.h``
  (``lib/libfe_kv_b200.so``; no fallback when it is missing).
* :mod:`fekv.ops`       the reference's ``fe::cuda`` operator interface
  (``create_plan``/``prepare_plan``/``attention``/``store``/``rope``/
  ``accept``) plus the fused ``rope_append`` and block copy.
* :mod:`fekv.metadata`  the per-step slot mapping / page tables of
  ``CudaModel::prepare``.
* :mod:`fekv.workloads` seeded synthetic configs C1..C5.
"""
from . import metadata, workloads  # noqa: F401
from ._lib import (FE_DTYPE_BF16, FE_DTYPE_F16, FeError, LIB_PATH, SHIM_PATH,  # noqa: F401
                   load)
from .ops import (AttentionPlan, HostPlan, accept, attention, clear_pages,  # noqa: F401
                  copy_blocks, create_plan, destroy_plan, device_errors, fork_copies, gather,
                  paged_decode_noalloc, prepare_plan, rope, rope_append, store)
