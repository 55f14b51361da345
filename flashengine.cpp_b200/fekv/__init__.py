"""fekv — host-side binding of the B200 paged-KV hot path.

* :mod:`fekv._lib`      ctypes binding of ``include/fe_kv.h``
  (``lib/libfe_kv_b200.so``; no fallback when it is missing).
* :mod:`fekv.ops`       the reference's ``fe::cuda`` operator interface
  (``create_plan``/``prepare_plan``/``attention``/``store``) plus block copy.
* :mod:`fekv.metadata`  the per-step slot mapping / page tables of
  ``CudaModel::prepare``.
* :mod:`fekv.workloads` seeded synthetic configs C1..C5.
"""
from . import metadata, workloads  # noqa: F401
from ._lib import (FE_DTYPE_BF16, FE_DTYPE_F16, FeError, LIB_PATH, SHIM_PATH,  # noqa: F401
                   load)
from .ops import (AttentionPlan, HostPlan, attention, clear_pages, copy_blocks,  # noqa: F401
                  create_plan, destroy_plan, device_errors, gather, paged_decode_noalloc,
                  prepare_plan, store)
