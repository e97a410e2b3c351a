"""Minimal stand-in for ``mlx_lm`` (fixture generation only)."""
