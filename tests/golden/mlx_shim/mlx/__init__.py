"""NumPy-backed stand-in for the ``mlx`` package (fixture generation only)."""
