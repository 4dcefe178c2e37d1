"""CPU float64 oracle for the rotor-scan hot path (test infrastructure only)."""
