"""CPU parity oracle (test infrastructure only; never imported by the eva_b200 package)."""
