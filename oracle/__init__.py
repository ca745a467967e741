"""CPU oracle for flash-Born attention (test infrastructure; never the product path)."""
