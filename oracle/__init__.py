"""CPU oracle for the quantized-linear path (test infrastructure only)."""
