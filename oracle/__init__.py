"""CPU oracle and coefficient derivation -- test infrastructure, not part of the product path."""
