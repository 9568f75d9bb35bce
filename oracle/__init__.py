"""CPU oracle for parity tests -- test infrastructure, never the product path."""
