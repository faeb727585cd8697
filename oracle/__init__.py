"""CPU oracle of the reference GGUF path (test infrastructure only; see gguf_oracle)."""
