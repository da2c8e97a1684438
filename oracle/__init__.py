"""CPU oracle of the reference's Dual-AR math (test infrastructure only)."""
