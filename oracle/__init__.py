"""CPU checkers for the quantized matrix path (test infrastructure only)."""
