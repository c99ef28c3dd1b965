"""CPU oracle for the tensor-product hot path: test infrastructure only (see o2_oracle)."""
