"""CPU oracle of the hot path (test infrastructure only; never imported by the product)."""
