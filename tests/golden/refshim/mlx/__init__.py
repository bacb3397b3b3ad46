"""CPU stand-in of the MLX modules the reference imports (test infrastructure only)."""
