"""CPU oracle of the decode operator (test infrastructure, never the product path)."""
