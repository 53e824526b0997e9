"""dtorch_b200 -- B200-native thread-group collectives behind DTorch's DTensor redistribute.

* ``capi``: ctypes binding of the C ABI (include/dtorch_b200.h) -- all-reduce (Partial->Replicate), all-gather
  (Shard->Replicate), reduce-scatter (Partial->Shard(0)) and all-to-all (Shard(i)->Shard(j)) as hand-written
  sm_100a kernels that move data through peer HBM over NVLink.
* ``DeviceMesh``, ``Shard``, ``Replicate``, ``Partial``, ``init_device_mesh``, ``DTensor`` (``redistribute``):
  the reference's Python API over the C++ host layer (``_host``: ThreadGroup, kernel-stream threads,
  redistribute executor).
"""

__version__ = "0.1.0"

_DTENSOR_NAMES = ("DeviceMesh", "Placement", "Shard", "Replicate", "Partial", "init_device_mesh", "DTensor",
                  "get_placements_from_dict",
                  "cuda_device_of", "clear", "redistribute_many", "reduce", "set_pool_bytes")


def __getattr__(name):
    if name in _DTENSOR_NAMES:
        from . import dtensor

        return getattr(dtensor, name)
    if name == "scaled_dot_product_attention_with_cp":
        from . import context_parallel

        return context_parallel.scaled_dot_product_attention_with_cp
    raise AttributeError(name)
