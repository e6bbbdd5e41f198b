"""CPU oracle (test infrastructure only): C restatement of the reference harness host code."""
