"""Routing math, row codecs, profiling and test helpers (pure torch, any device)."""
