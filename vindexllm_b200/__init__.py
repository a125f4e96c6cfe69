"""B200-native token sampler: drop-in for VindexLLM's TVdxSampler hot path."""
