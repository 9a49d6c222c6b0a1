"""Ming-Omni (BailingMM2): Whisper audio tower + BailingMoeV2 LLM."""
