"""fast_infer_b200: B200 (sm_100a) attention hot path of Fast_Infer.

Public surface (same names and semantics as the reference modules they replace):

* ``fast_infer_b200.kernels.attention.flash_attention`` / ``paged_attention``
  (reference kernels/attention.py)
* ``fast_infer_b200.kv_cache.KVCache`` plus ``store_kv_prefill`` / ``store_kv_decode``
  (reference kv_cache.py and model.py:162-201)
* ``fast_infer_b200.shard`` — KV-head / sequence partitioning across GPUs.

The compute runs in ``libfast_infer_b200.so`` (C ABI: include/fast_infer_b200.h).
"""

__version__ = "0.1.0"
