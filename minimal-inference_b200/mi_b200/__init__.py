"""B200-native paged-KV hot path for minimal-inference.

Host-side mirror of the reference's paged attention interface (FlashInfer's
``append_paged_kv_cache`` and the ``BatchDecode``/``BatchPrefill`` wrappers as
``model.py``/``scheduler.py`` call them), backed by hand-written sm_100a CUDA
kernels in ``libmi_paged.so`` (C ABI declared in ``include/mi_paged.h``).

Submodules are imported on demand; the CUDA library loads on first use and
raises if it is missing -- there is no CPU fallback.
"""

__all__ = [
    "capi", "page", "decode", "prefill", "kv_cache", "model", "scheduler",
    "rope", "weights", "glue", "tp_comm",
]
