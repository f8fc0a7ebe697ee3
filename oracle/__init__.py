"""CPU oracle of the Q4 fixed-point decode path (test infrastructure only)."""
