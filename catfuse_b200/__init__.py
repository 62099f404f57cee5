"""catfuse_b200 — B200-native (sm_100a) multi-step SNN inference hot path."""
__version__ = "0.1.0"
