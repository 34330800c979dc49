"""Stand-in for the `mlx_lm` package (test infrastructure; see ../README.md)."""
