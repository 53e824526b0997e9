"""dtorch_b200 -- B200-native thread-group collectives behind DTorch's DTensor redistribute.

The C ABI (include/dtorch_b200.h, ``capi``) is the drop-in boundary: all-reduce (Partial->Replicate),
all-gather (Shard->Replicate), reduce-scatter (Partial->Shard(0)) and all-to-all (Shard(i)->Shard(j)) as
hand-written sm_100a kernels that move data through peer HBM over NVLink.
"""

__version__ = "0.1.0"
