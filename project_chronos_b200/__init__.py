"""B200-native (sm_100a) Chronos MoE feed-forward layer."""
