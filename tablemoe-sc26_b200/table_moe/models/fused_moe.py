"""The cached MoE layer forward of the reference's wrappers on the ALUT kernels.

The reference's ``QwenMoeWrapperCached.forward`` (``qwen3_vl_moe/cached_layers.py:270-465``)
and its DeepSeek-VL2 counterpart (``deepseek_vl2/deepseek_layers.py:600-729``) run, per layer:

1. the router: ``qwen_topk_softmax`` and ``_build_compute_mask`` (``cached_layers.py:280-337``);
2. the expert loads and computations of the kept slots into ``collected_expert_outputs``;
3. the search of the other slots, then ``perform_value_fetch`` (``:340-351``): the hit ids are
   copied to the host (``.cpu()``, a device sync), the rows gathered from the pinned-host
   value table and copied back;
4. the combine (``:452-465``): hit rows written into ``collected_expert_outputs``, the
   routing weights renormalised over the survivors and a ``bmm``.

``ALUTCachedMoE`` keeps step 2 (the caller's experts) and replaces 1, 3 and 4 by three device
calls with no host round trip: ``alut_route`` (step 1), then one
``alut_lookup_combine_experts`` (search, gather from the HBM-resident value table,
renormalisation and the weighted sum of computed outputs and looked-up rows).
"""
from __future__ import annotations

import torch

from ..cache_engine import VectorSearchEngine
from ..ops.qwen_topk_softmax import route_for_lookup


class ALUTCachedMoE:
    """One MoE layer's routed-expert combine with ALUT lookups.

    ``run_experts(hidden_states, selected_experts, compute_mask, collected)`` must write the
    output of expert ``selected_experts[t, s]`` on token ``t`` into ``collected[t, s]`` for
    every slot with ``compute_mask[t, s]`` (the reference's expert loop writes
    ``collected_expert_outputs`` the same way); other rows are ignored.

    Defaults follow the Qwen3-VL wrapper: prefill keeps experts by importance
    (``KEEP_RATE``), decode keeps the first ``decode_keep_k`` slots; prefill searches with the
    dot rule (``search_prefill_offline_dot``), decode with the offline dot rule
    (``search_decode_offline_dot``); weights renormalised to one over the survivors.
    ``renorm="to_rowsum"`` gives the DeepSeek-VL2 rule.
    """

    def __init__(self, manager, top_k, *, normalize_topk=False, prefill_keep="importance", prefill_keep_k=3,
                 decode_keep_k=3, keep_rate=0.6, prefill_variant="prefill_dot", decode_variant="decode_dot",
                 renorm="to_one"):
        self.engine = VectorSearchEngine(manager)
        self.manager = manager
        self.top_k = int(top_k)
        self.normalize_topk = normalize_topk
        self.prefill_keep, self.prefill_keep_k = prefill_keep, prefill_keep_k
        self.decode_keep_k, self.keep_rate = decode_keep_k, keep_rate
        self.prefill_variant, self.decode_variant = prefill_variant, decode_variant
        self.renorm = renorm

    def route(self, router_logits, *, is_prefill, attn_scores=None):
        """(weights, selected_experts, compute_mask, reuse_mask) of ``_build_compute_mask``."""
        if is_prefill and self.prefill_keep == "importance":
            return route_for_lookup(router_logits, self.top_k, normalize_topk=self.normalize_topk, keep="importance",
                                    keep_rate=self.keep_rate, attn_scores=attn_scores)
        k = self.prefill_keep_k if is_prefill else self.decode_keep_k
        return route_for_lookup(router_logits, self.top_k, normalize_topk=self.normalize_topk, keep="fixed", keep_k=k)

    def __call__(self, hidden_states, router_logits, is_vision, run_experts, *, is_prefill, attn_scores=None,
                 return_routing=False):
        x = hidden_states.reshape(-1, hidden_states.shape[-1])
        w, sel, comp, reuse = self.route(router_logits, is_prefill=is_prefill, attn_scores=attn_scores)
        values = self.manager.values_buffer
        collected = torch.empty((x.shape[0], self.top_k, values.shape[-1]), dtype=values.dtype, device=x.device)
        run_experts(x, sel, comp, collected)
        out = self.engine.lookup_combine(x, sel, is_vision.reshape(-1), reuse, w, compute_mask=comp,
                                         variant=self.prefill_variant if is_prefill else self.decode_variant,
                                         renorm=self.renorm, computed=collected, return_hits=return_routing)
        if return_routing:
            out, hit, idx = out
            return out, dict(weights=w, selected_experts=sel, compute_mask=comp, reuse_mask=reuse, hit=hit, idx=idx)
        return out
