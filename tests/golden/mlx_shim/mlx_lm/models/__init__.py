"""Minimal stand-in for ``mlx_lm.models`` (fixture generation only)."""
