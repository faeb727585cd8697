"""GGUF block geometry and synthetic encoders (host side, numpy)."""
