"""CPU oracle of gs3d (test infrastructure only)."""
