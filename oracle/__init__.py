"""CPU oracle for the decoder token loop — test infrastructure only (see w4j_oracle.c)."""
