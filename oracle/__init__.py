"""CPU oracle for parity tests (test infrastructure only; never imported by the product)."""
