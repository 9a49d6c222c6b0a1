"""Stage executors of the Ming-Omni text pipeline:

  preprocessing -> audio_encoder -> mm_aggregate -> thinker -> decode

* preprocessing: Ming chat layout (``<role>SYSTEM</role>`` default system
  prompt + "detailed thinking off", ``<role>HUMAN</role>`` turns ended by
  ``<|role_end|>``, ``<role>ASSISTANT</role>`` generation prefix) with
  ``<audio>`` + one ``<audioPatch>`` per audio token + ``</audio>`` per audio
  (sglang_omni/models/ming_omni/components/preprocessor.py:206-290); audio is
  resampled to 16 kHz and passed on as a waveform;
* audio_encoder: log-mel on the GPU + the Whisper tower and projection;
* thinker: the paged engine over the BailingMoeV2 LLM, audio embeddings at
  the patch positions (the generic omni thinker stage);
* decode: final text.
"""
from __future__ import annotations

import torch

from ....engines.omni.factory import create_encoder_engine
from ....engines.omni.runtime.encoder import EncoderRequestData
from ....executors import EngineExecutor, PreprocessingExecutor
from ....ops.mel import LogMel
from ....proto import StagePayload
from ...qwen3_omni.pipeline import stages as qstages
from .. import loader
from ..hf_config import (AUDIO_END, AUDIO_PATCH, AUDIO_START, ROLE_ASSISTANT, ROLE_END, ROLE_HUMAN, ROLE_SYSTEM,
                         audio_tokens)

DEFAULT_SYSTEM_PROMPT = "你是一个友好的AI助手。"


def build_prompt(tok, messages, text, audio_counts: list[int]):
    """Returns (ids, audio_spans [(start, end)] of the <audioPatch> runs)."""
    parts = [f"{ROLE_SYSTEM}{DEFAULT_SYSTEM_PROMPT}\n\ndetailed thinking off{ROLE_END}"]
    msgs = list(messages or [])
    if msgs and msgs[0].get("role") == "system":
        parts[0] = f"{ROLE_SYSTEM}{msgs[0].get('content', DEFAULT_SYSTEM_PROMPT)}\n\ndetailed thinking off{ROLE_END}"
        msgs = msgs[1:]
    audio_block = "".join(f"{AUDIO_START}{AUDIO_PATCH * n}{AUDIO_END}" for n in audio_counts)
    if not msgs:
        msgs = [{"role": "user", "content": text or ""}]
    placed = False
    for m in msgs:
        tag = ROLE_HUMAN if m.get("role", "user") == "user" else ROLE_ASSISTANT
        c = m.get("content", "")
        if isinstance(c, list):
            c = "".join(x.get("text", "") if isinstance(x, dict) else str(x) for x in c)
        if tag == ROLE_HUMAN and not placed:
            c = audio_block + c
            placed = True
        parts.append(f"{tag}{c}{ROLE_END}")
    parts.append(ROLE_ASSISTANT)
    ids = tok.encode("".join(parts), add_special_tokens=False)
    patch = tok.convert_tokens_to_ids(AUDIO_PATCH)
    spans, i = [], 0
    while i < len(ids):
        if ids[i] == patch:
            j = i
            while j < len(ids) and ids[j] == patch:
                j += 1
            spans.append((i, j))
            i = j
        else:
            i += 1
    return ids, spans


def create_preprocessing_executor(model_path: str = "", overrides: dict | None = None):
    tok = loader.get_tokenizer(model_path, overrides)
    wcfg = loader._cfgs(model_path, overrides)["whisper"]

    def preprocess(payload: StagePayload) -> StagePayload:
        inp = payload.request.inputs if isinstance(payload.request.inputs, dict) else {}
        waves = [qstages._load_audio(a) for a in (inp.get("audios") or [])]
        counts = [audio_tokens(w.numel() // 160, wcfg) for w in waves]
        ids, spans = build_prompt(tok, inp.get("messages"), inp.get("prompt"), counts)
        p = torch.arange(len(ids), dtype=torch.int32)
        data = {"prompt_token_ids": ids, "audio_waveforms": waves, "audio_spans": spans,
                "images": [], "image_spans": [], "mrope_positions": torch.stack([p, p, p]), "mrope_delta": 0,
                "speech": False}
        return StagePayload(payload.request_id, payload.request, data)

    return PreprocessingExecutor(preprocess)


def create_audio_encoder_executor(model_path: str = "", device: str = "cuda:0", max_batch_size: int = 32,
                                  overrides: dict | None = None):
    dev = torch.device(device)
    enc = loader.get_audio_encoder(model_path, dev, overrides)
    mel = LogMel(enc.cfg.n_mels, dev)

    def encode(inputs: dict) -> list:
        per_req = inputs["waves"]
        flat = [w for ws in per_req for w in ws]
        mels = [mel(w.to(dev)) for w in flat]
        outs = enc(mels) if mels else []
        res, i = [], 0
        for ws in per_req:
            res.append({"audio_embeds": outs[i:i + len(ws)]})
            i += len(ws)
        return res

    engine = create_encoder_engine(encode, max_batch_size=max_batch_size, device=dev, cache_size=0)

    def request_builder(payload: StagePayload):
        waves = (payload.data or {}).get("audio_waveforms") or []
        return EncoderRequestData(inputs={"waves": waves}, skip=not waves)

    def result_builder(payload: StagePayload, out):
        if not isinstance(out, dict):
            out = {"audio_embeds": None}
        return StagePayload(payload.request_id, payload.request, out)

    return EngineExecutor(engine, request_builder, result_builder)


def create_thinker_executor(model_path: str = "", device: str = "cuda:0", max_batch: int = 64,
                            max_context: int = 8192, max_prefill_tokens: int = 8192, overrides: dict | None = None,
                            use_graphs: bool = True, thinker_max_seq_len: int | None = None):
    dev = torch.device(device)
    model = loader.get_llm(model_path, dev, overrides)
    return qstages.create_thinker_executor(model_path, device, max_batch,
                                           thinker_max_seq_len or max_context, max_prefill_tokens,
                                           overrides=overrides, use_graphs=use_graphs, model=model,
                                           tokenizer=loader.get_tokenizer(model_path, overrides),
                                           eos_token_ids=loader.eos_ids(model_path, overrides))


# the reference's factory name, so Ming configs written for it resolve
create_sglang_thinker_executor_from_config = create_thinker_executor
create_aggregate_executor = qstages.create_aggregate_executor
create_decode_executor = qstages.create_decode_executor
