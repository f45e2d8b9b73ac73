"""CPU oracle for the int4 path -- TEST INFRASTRUCTURE ONLY (see q4nx_oracle.c)."""
