"""Stage executors of the S2-Pro TTS pipeline:

  preprocessing (prompt + reference-audio DAC codes)
    -> tts_engine (batched dual-AR generation; streamed audio chunks for stream requests)
    -> vocoder (DAC decode of all codes; terminal)

Reference counterparts: create_preprocessing_executor / create_sglang_tts_engine_executor /
create_vocoder_executor and the incremental stream builder
(sglang_omni/models/fishaudio_s2_pro/pipeline/stages.py:100-409).

Streaming differs in where the work runs: the reference re-decodes every code
so far on the CPU after 5 and then every 100 tokens; here a vocoder thread
decodes on the GPU after ``stream_stride`` frames and then every
``stream_followup_stride`` frames.  ``stream_mode="stateful"`` (default) keeps
each stream's decoder state (``codec_stateful``): a chunk decodes only its new
frames and the chunks add up to the full decode exactly.  ``"window"`` re-decodes
a window of at most ``stream_context`` earlier frames before each chunk (the
decoder is causal, so a 48-frame context reproduces the full decode closely).
Ready streams are decoded together, one batched step per shape.
"""
from __future__ import annotations

import asyncio
import logging
import queue
import threading
import time
from collections import deque

import numpy as np
import torch

from ....executors import PreprocessingExecutor
from ....executors.interface import Executor, ResultQueueMixin
from ....executors.preprocessing_executor import StageError
from ....proto import StagePayload
from ....utils.hostdev import own_stream
from .. import loader
from ..generator import DualARGenerator, stream_seed
from ..tokenizer import Reference, S2ProPromptBuilder

log = logging.getLogger(__name__)

SPEECH_DEFAULTS = {"temperature": 0.8, "top_p": 0.8, "top_k": 30, "repetition_penalty": 1.1}


def _text_of(inputs) -> str:
    if isinstance(inputs, str):
        return inputs
    if not isinstance(inputs, dict):
        return ""
    if inputs.get("text") is not None:
        return str(inputs["text"])
    if inputs.get("prompt") is not None:
        return str(inputs["prompt"])
    for m in reversed(inputs.get("messages") or []):
        c = m.get("content") if isinstance(m, dict) else None
        if isinstance(c, str):
            return c
    return ""


# ----------------------------------------------------------------------------- preprocessing
def create_preprocessing_executor(model_path: str = "", overrides: dict | None = None, encode_device: str = "cpu"):
    tok = loader.get_tokenizer(model_path, overrides)
    cfg = loader.get_config(model_path, overrides)
    builder = S2ProPromptBuilder(tok, cfg.num_codebooks)

    def encode_reference(audio) -> torch.Tensor:
        from ....client.audio import decode_wav

        if isinstance(audio, str):
            with open(audio, "rb") as f:
                audio = f.read()
        if isinstance(audio, (bytes, bytearray)):
            wav, sr = decode_wav(bytes(audio))
        else:
            wav, sr = np.asarray(audio, dtype=np.float32), loader.dac_config(overrides).sample_rate
        x = torch.as_tensor(np.asarray(wav, dtype=np.float32)).reshape(-1)
        target = loader.dac_config(overrides).sample_rate
        if sr != target:
            n = int(round(x.numel() * target / sr))
            x = torch.nn.functional.interpolate(x[None, None], size=n, mode="linear", align_corners=False)[0, 0]
        enc = loader.get_encoder(model_path, encode_device, overrides)
        return enc.encode(x[None])[0].cpu()

    def preprocess(payload: StagePayload) -> StagePayload:
        req = payload.request
        inputs = req.inputs if req.inputs is not None else {}
        params = req.params or {}
        meta = req.metadata or {}
        text = _text_of(inputs)
        raw_refs = (inputs.get("references") if isinstance(inputs, dict) else None) or meta.get("references") or []
        refs = []
        for r in raw_refs:
            codes = r.get("vq_codes")
            if codes is not None:
                codes = torch.as_tensor(codes, dtype=torch.int32)
                if codes.dim() == 1:
                    codes = codes.view(cfg.num_codebooks, -1)
            elif r.get("audio_path") or r.get("audio") is not None:
                codes = encode_reference(r.get("audio_path") or r.get("audio"))
            refs.append(Reference(text=r.get("text") or "", vq_codes=codes))
        spk = meta.get("speaker", 0)
        prompt = builder.build(text, refs or None, speaker=spk if isinstance(spk, int) else 0)
        sp = dict(SPEECH_DEFAULTS)
        samp = params.get("sampling") or {}
        for k in ("temperature", "top_p", "top_k", "repetition_penalty", "seed", "ignore_eos"):
            if samp.get(k) is not None:
                sp[k] = samp[k]
        data = {
            "input_ids": prompt.ids,
            "vq_mask_tokens": prompt.vq_mask,
            "vq_parts": prompt.vq_codes.tolist(),
            "num_codebooks": cfg.num_codebooks,
            "codebook_size": cfg.codebook_size,
            "max_new_tokens": int(samp.get("max_new_tokens") or params.get("max_new_tokens") or 1024),
            **sp,
        }
        return StagePayload(payload.request_id, req, data)

    return PreprocessingExecutor(preprocess)


# ----------------------------------------------------------------------------- TTS engine
class S2ProTTSExecutor(ResultQueueMixin, Executor):
    """Runs the DualARGenerator on its own thread: admits requests (ragged
    prefill), advances every active request one frame per step, finishes on
    <|im_end|> or max_new_tokens.  Stream requests get audio chunks from a
    vocoder thread; the final payload carries all codes to the vocoder stage."""

    def __init__(self, model_path: str = "", device: str = "cuda:0", max_streams: int = 64, max_context: int = 4096,
                 max_new_tokens: int = 2048, overrides: dict | None = None, use_graphs: bool = True,
                 stream_stride: int = 5, stream_followup_stride: int = 20, stream_context: int = 48,
                 max_prefill_tokens: int = 8192, stream_mode: str = "stateful"):
        super().__init__()
        dev = torch.device(device)
        self.device = dev
        self.model_path = model_path
        self.overrides = overrides
        self.model = loader.get_model(model_path, dev, overrides)
        self.gen = DualARGenerator(self.model, max_streams=max_streams, max_context=max_context,
                                   use_graphs=use_graphs, max_prefill_tokens=max_prefill_tokens)
        self.max_new_tokens = max_new_tokens
        self.stream_stride = stream_stride
        self.stream_followup = stream_followup_stride
        self.stream_context = stream_context
        if stream_mode not in ("stateful", "window"):
            raise ValueError(f"stream_mode {stream_mode!r}: expected 'stateful' or 'window'")
        self.stream_mode = stream_mode
        self.max_streams = max_streams
        self._stateful = None    # StatefulStreamingDAC, built by _prepare_vocoder
        self._cv = threading.Condition()
        self._new: deque = deque()
        self._aborted: set[str] = set()
        self._pending: dict[str, dict] = {}
        self._codes: dict[str, list] = {}
        self._streams: dict[str, asyncio.Queue] = {}
        self._thread: threading.Thread | None = None
        self._voc_thread: threading.Thread | None = None
        self._voc_q: queue.Queue = queue.Queue()
        self._decoder = None
        self._loop: asyncio.AbstractEventLoop | None = None
        self._stop = False

    async def start(self):
        self._loop = asyncio.get_running_loop()
        if self.stream_mode == "stateful" and self.device.type == "cuda":
            # decoder weights, per-stream state and step graphs before the first request
            await asyncio.to_thread(self._prepare_vocoder)
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name="s2pro-tts", daemon=True)
            self._thread.start()

    async def stop(self):
        with self._cv:
            self._stop = True
            self._cv.notify_all()
        self._voc_q.put(None)

    async def add_request(self, payload: StagePayload) -> None:
        rid = payload.request_id
        params = payload.request.params or {}
        self._pending[rid] = {"payload": payload, "t0": time.perf_counter(), "stream": bool(params.get("stream")),
                              "emitted": 0, "next": self.stream_stride}
        if params.get("stream"):
            self._streams[rid] = asyncio.Queue()
        with self._cv:
            self._new.append(rid)
            self._cv.notify_all()

    def stream(self, request_id: str):
        q = self._streams.get(request_id)
        if q is None:
            return None

        async def gen():
            while True:
                item = await q.get()
                if item is None:
                    return
                yield item

        return gen()

    async def abort(self, request_id: str) -> None:
        with self._cv:
            self._aborted.add(request_id)
            self._cv.notify_all()
        q = self._streams.pop(request_id, None)
        if q is not None:
            q.put_nowait(None)

    # ------------------------------------------------------------------ threads
    def _post(self, fn, *a):
        if self._loop is not None:
            self._loop.call_soon_threadsafe(fn, *a)

    def _finish(self, rid: str, error: str | None = None):
        info = self._pending.pop(rid, None)
        codes = self._codes.pop(rid, [])
        if info is None:
            return
        p = info["payload"]
        if error is not None:
            self._post(self._results().put_nowait, StageError(rid, error))
            self._close_stream(rid)
            return
        arr = np.asarray(codes, dtype=np.int64).T if codes else np.zeros((self.gen.ncb + 1, 0), np.int64)
        d = dict(p.data)
        d.update({"output_codes": arr.tolist(), "prompt_tokens": len(p.data.get("input_ids") or []),
                  "completion_tokens": int(arr.shape[1]), "engine_time_s": time.perf_counter() - info["t0"]})
        if info["stream"]:
            self._voc_q.put((rid, codes, info, True))
        self._post(self._results().put_nowait, StagePayload(rid, p.request, d))

    def _close_stream(self, rid: str):
        q = self._streams.pop(rid, None)
        if q is not None:
            self._post(q.put_nowait, None)
        if self._stateful is not None:
            self._voc_q.put((rid, None, None, True))   # frees the stream's decoder slot

    def _run(self):
        stream = own_stream(self.device)
        if stream is not None:
            torch.cuda.set_stream(stream)
        try:
            with torch.inference_mode():
                self.gen.capture_all()
                self._loop_body()
        except BaseException as exc:  # the engine thread died: fail every request it holds
            log.exception("s2pro engine thread failed")
            for rid in list(self._pending):
                self._finish(rid, error=f"tts_engine failed: {exc}")

    def _admit(self, rids: list[str]) -> list:
        out = []
        gen = self.gen
        for rid in rids:
            info = self._pending.get(rid)
            if info is None:
                continue
            d = info["payload"].data
            ids = list(d["input_ids"])
            mask = torch.tensor(d.get("vq_mask_tokens") or [False] * len(ids), dtype=torch.bool)
            rows = torch.full((len(ids),), -1, dtype=torch.int32)
            rows[mask] = torch.arange(int(mask.sum()), dtype=torch.int32)
            vq = torch.as_tensor(d.get("vq_parts") or [], dtype=torch.int32).reshape(-1, gen.ncb)
            seed = d.get("seed")
            try:
                out.append(gen.add_stream(rid, ids, rows, vq, min(int(d.get("max_new_tokens") or 1024),
                                                                    self.max_new_tokens),
                                          float(d.get("temperature", 0.8)), float(d.get("top_p", 0.8)),
                                          int(d.get("top_k", 30)), float(d.get("repetition_penalty", 1.1)),
                                          int(seed) if seed is not None else stream_seed(rid) & ((1 << 62) - 1)))
                self._codes[rid] = []
            except (ValueError, RuntimeError) as exc:
                self._finish(rid, error=f"tts_engine: {exc}")
        return out

    def _emit(self, streams, codes: torch.Tensor):
        host = codes.cpu().tolist()
        im_end = self.model.cfg.im_end_id
        for s, c in zip(streams, host):
            info = self._pending.get(s.rid)
            if c[0] == im_end and not (info is not None and info["payload"].data.get("ignore_eos")):
                s.finished = True
            else:
                self._codes.setdefault(s.rid, []).append(c)
                if s.frames >= s.max_new_tokens:
                    s.finished = True
            if info is not None and info["stream"] and not s.finished:
                n = len(self._codes[s.rid])
                if n >= info["next"]:
                    info["next"] = n + self.stream_followup
                    self._voc_q.put((s.rid, list(self._codes[s.rid]), info, False))
            if s.finished:
                self._finish(s.rid)
                self.gen.remove(s.rid)

    def _loop_body(self):
        gen = self.gen
        self._voc_thread = threading.Thread(target=self._vocoder_loop, name="s2pro-stream-vocoder", daemon=True)
        self._voc_thread.start()
        while True:
            with self._cv:
                while not self._stop and not self._new and not self._aborted and not gen.active():
                    self._cv.wait(timeout=0.5)
                if self._stop:
                    return
                aborted, self._aborted = self._aborted, set()
                new = []
                while self._new and len(new) < len(gen.free_slots):
                    new.append(self._new.popleft())
            for rid in aborted:
                gen.remove(rid)
                self._pending.pop(rid, None)
                self._codes.pop(rid, None)
                if self._stateful is not None:
                    self._voc_q.put((rid, None, None, True))
            new = [r for r in new if r not in aborted]
            streams = self._admit(new)
            # ragged prefill in groups that fit the prefill budget
            group, tokens = [], 0
            for s in streams + [None]:
                if s is None or (group and tokens + len(s.prompt_ids) > gen.max_prefill_tokens):
                    if group:
                        self._emit(group, gen.prefill(group))
                    group, tokens = [], 0
                if s is not None:
                    group.append(s)
                    tokens += len(s.prompt_ids)
            ready = gen.active()
            if ready:
                self._emit(ready, gen.step(ready))

    def _vocoder_loop(self):
        """Decodes the stream windows of every stream with a chunk ready, batched:
        one decoder forward per (window length, context) group."""
        stream = own_stream(self.device)
        if stream is not None:
            torch.cuda.set_stream(stream)  # chunks do not wait behind generation steps
        while True:
            jobs = [self._voc_q.get()]
            while True:
                try:
                    jobs.append(self._voc_q.get_nowait())
                except queue.Empty:
                    break
            stop = any(j is None for j in jobs)
            latest: dict[str, tuple] = {}
            finals: set[str] = set()
            closed: set[str] = set()
            for j in jobs:
                if j is None:
                    continue
                rid, codes, info, final = j
                if codes is None:          # the stream ended or was aborted: release its state
                    closed.add(rid)
                    continue
                if rid not in latest or len(codes) >= len(latest[rid][0]):
                    latest[rid] = (codes, info)
                if final:
                    finals.add(rid)
            try:
                if self.stream_mode == "stateful":
                    self._decode_stateful(latest, finals)
                else:
                    self._decode_batch(latest)
            except Exception:
                log.exception("stream vocoding failed")
            for rid in finals:
                self._close_stream(rid)
            if self._stateful is not None:
                for rid in closed:
                    self._stateful.close(rid)
            if stop:
                return

    def _prepare_vocoder(self):
        """The stateful stream decoder: DAC weights, one state slot per generator stream, and
        (on a GPU) the step graphs of the first chunk and the follow-up chunks."""
        if self._stateful is not None:
            return
        from ..codec_stateful import StatefulStreamingDAC

        if self._decoder is None:
            self._decoder = loader.get_decoder(self.model_path, self.device, self.overrides)
        sd = StatefulStreamingDAC(self._decoder, chunk=self.stream_followup, first_chunk=self.stream_stride,
                                  max_streams=self.max_streams)
        with torch.inference_mode():
            sd.capture_graphs()
        self._stateful = sd

    def _decode_stateful(self, latest: dict[str, tuple], finals: set[str]):
        if not latest:
            return
        self._prepare_vocoder()
        sd = self._stateful
        for rid, (codes, _) in latest.items():
            have = sd.frames(rid)
            if len(codes) > have:
                sd.add_codes(rid, torch.tensor(codes[have:], dtype=torch.long)[:, 1:])
        with torch.inference_mode():
            out = sd.decode_ready(list(latest), finals=finals, to_host=True)
        now = time.perf_counter()
        rate = self._decoder.cfg.sample_rate
        for rid, a in out.items():
            info = latest[rid][1]
            info["emitted"] += a.size
            q = self._streams.get(rid)
            if q is not None and a.size:
                self._post(q.put_nowait, {"modality": "audio", "audio_waveform": a, "sample_rate": rate, "t": now})

    def _decode_batch(self, latest: dict[str, tuple]):
        if not latest:
            return
        if self._decoder is None:
            self._decoder = loader.get_decoder(self.model_path, self.device, self.overrides)
        dec = self._decoder
        hop = dec.cfg.hop
        groups: dict[tuple[int, int], list] = {}
        for rid, (codes, info) in latest.items():
            n = len(codes)
            done = info["emitted"] // hop
            if n <= done:
                continue
            start = max(0, done - self.stream_context)
            groups.setdefault((n - start, done - start), []).append((rid, codes[start:n], info, n))
        for (_, ctx), items in groups.items():
            win = torch.tensor([c for _, c, _, _ in items], dtype=torch.int64)[:, :, 1:]   # [B, W, ncb]
            with torch.inference_mode():
                wav = dec.decode(win.permute(0, 2, 1).contiguous().to(self.device))
            wav = wav[:, ctx * hop:].float().cpu().numpy()
            now = time.perf_counter()
            for (rid, _, info, n), a in zip(items, wav):
                info["emitted"] = n * hop
                q = self._streams.get(rid)
                if q is not None and a.size:
                    self._post(q.put_nowait, {"modality": "audio", "audio_waveform": a,
                                              "sample_rate": dec.cfg.sample_rate, "t": now})


def create_tts_engine_executor(model_path: str = "", device: str = "cuda:0", max_new_tokens: int = 2048,
                               max_streams: int = 64, max_context: int = 4096, overrides: dict | None = None,
                               use_graphs: bool = True, stream_stride: int = 5, stream_followup_stride: int = 20,
                               stream_context: int = 48, top_k: int | None = None, stream_mode: str = "stateful"):
    """Same factory arguments as the reference (device, max_new_tokens, stream strides);
    ``stream_mode``: "stateful" (kept decoder state per stream) or "window"."""
    return S2ProTTSExecutor(model_path, device, max_streams, max_context, max_new_tokens, overrides, use_graphs,
                            stream_stride, stream_followup_stride, stream_context, stream_mode=stream_mode)


# alias of the reference's factory name, so configs written for it resolve
create_sglang_tts_engine_executor = create_tts_engine_executor


# ----------------------------------------------------------------------------- vocoder
def create_vocoder_executor(model_path: str = "", device: str = "cuda:0", overrides: dict | None = None):
    dev = torch.device(device)
    dec = loader.get_decoder(model_path, dev, overrides)
    lock = threading.Lock()

    def vocode(payload: StagePayload) -> StagePayload:
        d = dict(payload.data)
        codes = torch.as_tensor(d.get("output_codes") or [], dtype=torch.int64)
        if codes.numel():
            with lock, torch.inference_mode():
                wav = dec.decode(codes[1:].to(dev)[None])[0].float().cpu().numpy()
        else:
            wav = np.zeros(0, np.float32)
        d["audio_waveform"] = wav
        d["sample_rate"] = dec.cfg.sample_rate
        d["modality"] = "audio"
        pt, ct = int(d.get("prompt_tokens") or 0), int(d.get("completion_tokens") or 0)
        usage = {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct}
        if d.get("engine_time_s"):
            usage["engine_time_s"] = round(float(d["engine_time_s"]), 6)
        d["usage"] = usage
        d.pop("vq_parts", None)
        return StagePayload(payload.request_id, payload.request, d)

    return PreprocessingExecutor(vocode)
