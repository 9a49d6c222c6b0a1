"""Module paths of the reference's Qwen3-Omni component executors
(sglang_omni/models/qwen3_omni/components/), so its pipeline configs resolve."""
