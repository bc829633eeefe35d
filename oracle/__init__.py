"""CPU oracle for the sampling path (test infrastructure; see sampler_oracle)."""
