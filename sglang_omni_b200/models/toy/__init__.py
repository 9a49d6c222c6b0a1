"""Two-stage toy pipeline: identity preprocessing -> tiny Llama-style decoder (CPU, fp32)."""
