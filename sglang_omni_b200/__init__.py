"""sglang_omni_b200: a B200-native (sm_100a) multi-stage omni-model serving runtime.

Layers (bottom-up): ops (sm_100a kernels) -> models -> engines (paged AR,
encoder) -> executors -> pipeline (coordinator, stages, workers, relay) ->
config -> client -> serve (OpenAI-compatible HTTP) -> cli.
"""
__version__ = "0.1.0"
