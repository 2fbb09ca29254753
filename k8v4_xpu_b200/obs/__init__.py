"""Observability: stage profiler, attention timer (opt-in, off the hot path when disabled)."""
