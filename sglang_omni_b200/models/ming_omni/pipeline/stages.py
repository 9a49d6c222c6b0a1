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

import asyncio
import logging
import threading
from collections import deque

import torch

from ....engines.omni.factory import create_encoder_engine
from ....engines.omni.runtime.encoder import EncoderRequestData
from ....executors import EngineExecutor, PreprocessingExecutor
from ....executors.interface import Executor, ResultQueueMixin
from ....ops.mel import LogMel
from ....executors.preprocessing_executor import StageError
from ....proto import StagePayload
from ...qwen3_omni.pipeline import stages as qstages
from .. import loader
from ..hf_config import (AUDIO_END, AUDIO_PATCH, AUDIO_START, ROLE_ASSISTANT, ROLE_END, ROLE_HUMAN, ROLE_SYSTEM,
                         audio_tokens)

DEFAULT_SYSTEM_PROMPT = "你是一个友好的AI助手。"


log = logging.getLogger(__name__)

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
        mels = mel.batch(flat) if flat else []
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


# ----------------------------------------------------------------------------- talker (speech output)
class MingTalkerExecutor(ResultQueueMixin, Executor):
    """Speech from the thinker's text: every request becomes a talker stream; one
    generator thread steps all live streams in lock step (one CUDA graph per
    step and batch bucket) and decodes each finished stream's latents with the
    AudioVAE.  The result carries ``audio_waveform`` / ``sample_rate`` /
    ``duration`` (reference: MingTalkerExecutor,
    sglang_omni/models/ming_omni/components/talker_executor.py:34-308)."""

    def __init__(self, model_path: str, device: str, max_streams: int = 32, max_patches: int = 256,
                 overrides: dict | None = None, use_graphs: bool = True, cfg_strength: float = 2.0,
                 voice: str | None = None):
        super().__init__()
        from ..talker import MingSpeechGenerator

        dev = torch.device(device)
        self.device = dev
        self.talker = loader.get_talker(model_path, dev, overrides)
        self.vae = loader.get_audio_vae(model_path, dev, overrides)
        self.tok = loader.get_talker_tokenizer(model_path, overrides)
        self.gen = MingSpeechGenerator(self.talker, max_streams=max_streams, cfg_strength=cfg_strength,
                                       use_graphs=use_graphs and dev.type == "cuda")
        self.max_patches = max_patches
        self.voice = voice
        self._cv = threading.Condition()
        self._new: deque = deque()
        self._aborted: set[str] = set()
        self._pending: dict[str, StagePayload] = {}
        self._thread: threading.Thread | None = None
        self._loop: asyncio.AbstractEventLoop | None = None
        self._stop = False
        self.error: BaseException | None = None

    async def start(self):
        self._loop = asyncio.get_running_loop()
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name="ming-talker", daemon=True)
            self._thread.start()

    async def stop(self):
        with self._cv:
            self._stop = True
            self._cv.notify_all()

    @staticmethod
    def _text_of(data: dict) -> str:
        for k in ("text", "generated_text"):
            if data.get(k):
                return str(data[k])
        return str((data.get("stream_state") or {}).get("accumulated_text", ""))

    async def add_request(self, payload: StagePayload) -> None:
        if self._loop is None:
            await self.start()
        text = self._text_of(payload.data or {})
        self._pending[payload.request_id] = payload
        if self.error is not None:
            self._deliver(payload.request_id, None, error=f"talker failed: {self.error}")
            return
        if not text.strip():
            self._deliver(payload.request_id, None)
            return
        with self._cv:
            self._new.append((payload.request_id, text))
            self._cv.notify_all()

    async def abort(self, request_id: str) -> None:
        with self._cv:
            self._aborted.add(request_id)
            self._cv.notify_all()

    def _deliver(self, rid: str, wav, error: str | None = None):
        p = self._pending.pop(rid, None)
        if p is None:
            return
        if error is not None:
            item = StageError(rid, error)
        else:
            sr = self.vae.cfg.sample_rate
            n = 0 if wav is None else int(wav.shape[-1])
            item = StagePayload(rid, p.request, {"audio_waveform": wav, "sample_rate": sr, "duration": n / sr,
                                                 "modality": "audio"})
        self._loop.call_soon_threadsafe(self._results().put_nowait, item)

    def _prefill_embeds(self, text: str) -> torch.Tensor:
        from ..talker import build_talker_prompt

        ids, _rows = build_talker_prompt(self.tok, text)
        lm = self.talker.lm
        idx = torch.tensor(ids, dtype=torch.long, device=self.device)
        return lm.embed[idx]

    def _run(self):
        from ....utils.hostdev import own_stream

        stream = own_stream(self.device)
        if stream is not None:
            torch.cuda.set_stream(stream)
        try:
            with torch.inference_mode():
                self.gen.capture_all()
                self._loop_body()
        except BaseException as exc:  # fail every request of this stage, now and later
            log.exception("Ming talker thread failed")
            self.error = exc
            for rid in list(self._pending):
                self._deliver(rid, None, error=f"talker failed: {exc}")

    def _loop_body(self):
        live: dict = {}
        while True:
            with self._cv:
                while not self._new and not live and not self._stop:
                    self._cv.wait(timeout=0.5)
                if self._stop:
                    return
                new, self._new = list(self._new), deque()
                aborted, self._aborted = set(self._aborted), set()
            for rid in aborted:
                if rid in live:
                    self.gen.remove(rid)
                    live.pop(rid)
                self._pending.pop(rid, None)
            fresh = []
            for rid, text in new:
                if rid in aborted:
                    continue
                if len(live) + len(fresh) >= self.gen.max_streams:
                    with self._cv:
                        self._new.appendleft((rid, text))
                    continue
                st = self.gen.add_stream(rid, self._prefill_embeds(text), max_patches=self.max_patches)
                fresh.append(st)
                live[rid] = st
            if fresh:
                self.gen.prefill(fresh)
            run = [s for s in live.values() if not s.done]
            if run:
                self.gen.step(run)
            for rid, st in list(live.items()):
                if st.done:
                    lat = torch.stack(st.latents, 0).reshape(-1, self.talker.cfg.latent_dim)
                    wav = self.vae.decode(lat.unsqueeze(0).to(self.device))[0].float().cpu().numpy()
                    self.gen.remove(rid)
                    live.pop(rid)
                    self._deliver(rid, wav)


def create_talker_executor(model_path: str = "", device: str = "cuda:0", voice: str | None = None,
                           max_streams: int = 32, max_patches: int = 256, overrides: dict | None = None,
                           use_graphs: bool = True, talker_model_path: str | None = None):
    """The Ming TTS talker stage (own Qwen2 LM + CFM/DiT + aggregator + AudioVAE)."""
    return MingTalkerExecutor(talker_model_path or model_path, device, max_streams=max_streams,
                              max_patches=max_patches, overrides=overrides, use_graphs=use_graphs, voice=voice)
