"""CPU restatement of the reference mixer path — test infrastructure only."""
