"""Process-wide cache configuration, read as ``CacheConfig.NAME``.

Same keys, defaults and update functions as the reference's
``table_moe/cache_engine/config.py:12-74``: the model builders set it per model and the
search engine reads the thresholds from it at call time.
"""
from __future__ import annotations

import os
from pathlib import Path

import torch

DEFAULT_OFFLINE_ROOT = Path(os.getenv("TABLEMOE_OFFLINE_ROOT", "offline_table/ds_fp16"))
DEFAULT_BENCHMARK = "MMBench_DEV_EN_V11"


def _defaults() -> dict:
    return {
        "PCA_DIR": os.getenv(
            "DS_CACHE_PCA_DIR",
            str(DEFAULT_OFFLINE_ROOT / "clustering_results" / f"{DEFAULT_BENCHMARK}_LayerPCA_256")),
        "CACHE_DIR": os.getenv(
            "DS_CACHE_DIR",
            str(DEFAULT_OFFLINE_ROOT / "offline_table" / f"{DEFAULT_BENCHMARK}_LayerPCA_256")),
        "COMPRESSED_DIM": 64,
        "FIXED_K": 256,
        "KEEP_K": 3,
        "PREFILL_KEEP_K": 3,
        "DECODE_KEEP_K": 3,
        "KEEP_RATE": 0.6,
        "MODALITY_MAP": {"vision": 0, "text": 1},
        "ONLINE_CACHE_SIZE": 64,
        "ONLINE_TOP_K": 6,
        "ONLINE_MIN_LAYER_IDX": 1,
        "ONLINE_MAX_LAYER_IDX": 47,
        "MODEL_DTYPE": torch.bfloat16,
        "OFFLINE_COSINE_THRESHOLD_VISION": 0.6,
        "OFFLINE_COSINE_THRESHOLD_TEXT": 0.7,
        "OFFLINE_DOT_THRESHOLD": 0.0,
        "OFFLINE_COSINE_EPS": 1e-6,
        # Not in the reference: read the kernels' device error bits after every search
        # (synchronises the stream; raises IndexError for out-of-range expert ids, as the
        # reference's indexing does, and RuntimeError for timed-out device waits).
        "ALUT_CHECK_ERRORS": os.getenv("TABLEMOE_ALUT_CHECK_ERRORS", "0") == "1",
    }


_active = _defaults()


def set_active_cache_config(config):
    """Replace the active config by the defaults updated with `config`."""
    global _active
    fresh = _defaults()
    if config is not None:
        fresh.update(config)
    _active = fresh


def update_active_cache_config(**kwargs):
    _active.update(kwargs)


def get_active_cache_config():
    return dict(_active)


class _Meta(type):
    def __getattr__(cls, name):
        try:
            return _active[name]
        except KeyError:
            raise AttributeError(name) from None

    def __setattr__(cls, name, value):
        if name in _active:
            _active[name] = value
        else:
            super().__setattr__(name, value)


class CacheConfig(metaclass=_Meta):
    """Attribute view of the active configuration (``CacheConfig.FIXED_K`` ...)."""
