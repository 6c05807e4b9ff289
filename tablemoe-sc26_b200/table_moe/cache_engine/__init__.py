from .config import CacheConfig, get_active_cache_config, set_active_cache_config, update_active_cache_config
from .manager import HybridStorageManager
from .search import HAS_TRITON, VectorSearchEngine

__all__ = [
    "CacheConfig",
    "get_active_cache_config",
    "HybridStorageManager",
    "HAS_TRITON",
    "set_active_cache_config",
    "update_active_cache_config",
    "VectorSearchEngine",
]
