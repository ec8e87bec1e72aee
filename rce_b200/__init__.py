"""rce_b200 -- B200-native (sm_100a) GGUF block-quantized matmul for the
Q8_0, Q4_0, Q4_K, Q5_K and Q6_K formats, a drop-in for the reference crate rce-op-qmm's
operator API.  Compute runs in librce_qmm.so (include/rce_qmm.h); this
package is the host-side mirror of the reference interface."""
from .gguf import GgufDtype, GgufFile, GgufParseError, tensor_byte_size  # noqa: F401
from .qmm import (  # noqa: F401
    Context,
    CudaQmm,
    QmmError,
    QmmLeaf,
    QuantWeight,
    Unsupported,
    default_context,
    dequant_device,
    mm_1d,
    mm_1d_serial,
    mm_batched,
    mm_batched_device,
    mm_multi_device,
)
from .moe import (RouterDecision, decisions, moe_ffn, moe_ffn_device, moe_route_device, moe_router,  # noqa: F401
                  moe_router_device, moe_shared_expert_device, split_experts)
from .shard import PeerGroup, row_shards, torch_exchange  # noqa: F401

__version__ = "0.1.0"
