"""CPU oracle for the IMI path (test infrastructure; never imported by the product)."""
