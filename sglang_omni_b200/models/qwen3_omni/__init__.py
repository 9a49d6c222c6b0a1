"""Qwen3-Omni-30B-A3B: thinker, talker, code predictor, code2wav, audio / vision encoders."""
