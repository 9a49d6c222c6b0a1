"""Stage factories shared by the text pipelines: chat / prompt preprocessing
(tokenise, chat template) and the routing helpers."""
from __future__ import annotations

from typing import Any

from ...executors import PreprocessingExecutor
from ...proto import StagePayload
from .tokenizer import load_tokenizer


def tokenize_inputs(tokenizer, inputs: Any) -> list[int]:
    if isinstance(inputs, dict):
        if inputs.get("prompt_token_ids") is not None:
            return list(inputs["prompt_token_ids"])
        if inputs.get("messages"):
            ids = tokenizer.apply_chat_template(inputs["messages"], add_generation_prompt=True, tokenize=True)
            return list(ids["input_ids"] if isinstance(ids, dict) else ids)
        if inputs.get("prompt") is not None:
            return list(tokenizer.encode(inputs["prompt"]))
    if isinstance(inputs, (list, tuple)):
        return list(inputs)
    if isinstance(inputs, str):
        return list(tokenizer.encode(inputs))
    raise ValueError("request has no prompt, messages or prompt_token_ids")


def create_text_preprocessing_executor(model_path: str = "", vocab_size: int = 151936):
    tok = load_tokenizer(model_path, vocab_size)

    def preprocess(payload: StagePayload) -> StagePayload:
        ids = tokenize_inputs(tok, payload.request.inputs if payload.data is None else payload.data)
        return StagePayload(payload.request_id, payload.request, {"prompt_token_ids": ids})

    return PreprocessingExecutor(preprocess)


def create_identity_executor(inject_faults: list | None = None, **_):
    """Passes payloads through.  ``inject_faults``: control-plane fault rules
    (``pipeline.faults.FaultRule`` fields) installed in this stage's process (tests)."""
    if inject_faults:
        from ...pipeline import faults

        faults.inject([faults.FaultRule(**r) for r in inject_faults])
    return PreprocessingExecutor(lambda p: p)


def terminal(request_id: str, payload: StagePayload):
    return None
