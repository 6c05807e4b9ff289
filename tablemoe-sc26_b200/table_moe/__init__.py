"""B200-native ALUT path of TableMoE.

Only ``table_moe.cache_engine`` is provided here: it is a drop-in replacement for the
reference's ``table_moe/cache_engine`` package (same module, class and method names and
arguments), whose search, gather and combine run on hand-written sm_100a kernels.
"""
