"""ExpertFlow MoE-layer hot path on B200 (sm_100a)."""
