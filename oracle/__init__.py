"""CPU oracle for the RoPE + KV-append path: test infrastructure, never the product path."""
