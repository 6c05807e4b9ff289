"""Router op of the TableMoE layers on sm_100a (drop-in for the reference's
``table_moe/ops`` entry ``qwen_topk_softmax``; the fp16 fused expert MLP of that package is
not part of the lookup path and is not provided)."""
from .qwen_topk_softmax import qwen_topk_softmax, route_for_lookup

__all__ = ["qwen_topk_softmax", "route_for_lookup"]
