"""CPU oracle (test infrastructure only; see oracle/ref_cpu.c)."""
