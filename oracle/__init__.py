"""CPU oracle for the MoC hot path — test infrastructure only (see moc_oracle.py)."""
