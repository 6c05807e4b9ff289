"""B200-native ALUT path of TableMoE.

Drop-in packages for the reference's lookup path: ``table_moe.cache_engine`` (search,
gather, combine), ``table_moe.ops.qwen_topk_softmax`` (router top-k softmax) and
``table_moe.skip`` (keep masks), with the same module, function, class and method names and
arguments as the reference; the work runs on hand-written sm_100a kernels.
"""
