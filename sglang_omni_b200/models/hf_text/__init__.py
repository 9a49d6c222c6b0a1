"""Any Hugging Face dense (or Qwen3-MoE) causal language model on the paged engine:
``decoder_from_hf`` converts a transformers model or a local checkpoint directory into a
``DecoderLM``; ``config.HFTextPipelineConfig`` serves it as a two-stage text pipeline."""
from .convert import SUPPORTED_ARCHITECTURES, decoder_config_from_hf, decoder_from_hf

__all__ = ["SUPPORTED_ARCHITECTURES", "decoder_config_from_hf", "decoder_from_hf"]
