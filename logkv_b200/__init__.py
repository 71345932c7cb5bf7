"""B200-native SemanticLogKV flush-and-attend path (sm_100a CUDA behind a C-ABI library)."""
