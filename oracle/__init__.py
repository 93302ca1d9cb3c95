"""CPU oracle (test infrastructure only): restatement of the reference MoE path in numpy."""
