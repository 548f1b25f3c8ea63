"""rotatek_b200 (package init written later)."""
