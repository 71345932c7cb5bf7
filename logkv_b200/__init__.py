"""B200-native SemanticLogKV flush-and-attend path (sm_100a CUDA behind a C-ABI library)."""
from .attention import log_kv_chunk_attention, pack_mid_kv  # noqa: F401
from .cache import LogStructuredKVCache, _SemanticReplayUpdates  # noqa: F401
