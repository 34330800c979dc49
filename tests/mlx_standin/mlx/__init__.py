"""Stand-in for the `mlx` package (test infrastructure; see ../README.md)."""
