"""CPU oracle of the Ulysses attention path (test infrastructure only)."""
