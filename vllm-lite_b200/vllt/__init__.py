"""vllt: a B200-native (sm_100a) forward hot path for vllm-lite-style serving."""
