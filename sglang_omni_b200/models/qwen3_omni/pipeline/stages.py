"""Stage factories of the Qwen3-Omni pipelines.

preprocessing  (CPU)  chat layout with audio / image placeholders, M-RoPE positions
audio_encoder  (GPU)  batched log-mel + audio tower (generic step engine, LRU cache)
image_encoder  (GPU)  vision tower (skips requests without images)
mm_aggregate          fan-in -> thinker input
thinker        (GPU)  paged AR engine; text deltas to the client; in speech mode
                      every token (and the prompt's accept-layer states) is
                      streamed to talker_ar
decode                terminal text result
talker_ar      (GPU)  SpeechGenerator: talker + code predictor for all streams
                      in lock step, code frames streamed to code2wav
code2wav       (GPU)  streaming vocoder, audio chunks to the client

Reference counterpart: sglang_omni/models/qwen3_omni/pipeline/stages.py:56-675
and the streaming executors in sglang_omni/models/qwen3_omni/components/.
"""
from __future__ import annotations

import asyncio
import base64
import io
import logging
import os
import threading
import time
from collections import deque
from typing import Any

import numpy as np
import torch

from ....engines.ar import AREngine, ARRequest, KVPool
from ....engines.ar.adapter import PagedAREngineAdapter
from ....engines.omni.factory import create_encoder_engine
from ....engines.omni.runtime.encoder import EncoderRequestData
from ....executors import EngineExecutor, PreprocessingExecutor
from ....executors.interface import Executor, ResultQueueMixin
from ....executors.preprocessing_executor import StageError
from ....pipeline import fastlane
from ....ops.mel import LogMel
from ....utils import trace
from ....proto import StagePayload
from ....utils.hostdev import adopt, h2d, own_stream
from ...common.ar_stage import sampling_for
from ...common.tokenizer import IncrementalDetokenizer, load_tokenizer
from .. import loader
from ..engine_io import build_prompt, mrope_positions
from ..hf_config import THINKER_EOS_IDS
from ..talker import SpeechGenerator, build_talker_prefill
from ..code2wav import Code2WavGraphs, StreamingCode2Wav
from ..code2wav_stateful import StatefulStreamingCode2Wav

log = logging.getLogger(__name__)
SAMPLE_RATE_IN = 16000
SAMPLE_RATE_OUT = 24000


def _speech_requested(params: dict) -> bool:
    mods = params.get("output_modalities") or []
    return "audio" in mods or params.get("task") == "tts"


# ----------------------------------------------------------------------------- preprocessing
def _load_image(item: Any) -> np.ndarray:
    """uint8 RGB [H, W, 3] from an array / nested list / PIL image / path / base64 (PNG/JPEG via PIL)."""
    if isinstance(item, dict):
        item = item.get("url") or item.get("image") or item.get("data")
    if isinstance(item, (str, bytes, bytearray)):
        from PIL import Image

        from ....preprocessing.media import fetch, is_url

        if isinstance(item, (bytes, bytearray)):
            raw = bytes(item)
        elif is_url(item) or os.path.exists(item):
            raw = fetch(item)
        else:
            raw = base64.b64decode(item, validate=True)
        item = np.asarray(Image.open(io.BytesIO(raw)).convert("RGB"))
    arr = np.asarray(item)
    if arr.dtype != np.uint8:
        arr = np.clip(arr, 0, 255).astype(np.uint8)
    if arr.ndim == 2:
        arr = np.repeat(arr[..., None], 3, -1)
    return arr


def _load_audio(item: Any) -> torch.Tensor:
    """Waveform at 16 kHz from an array / list / {"array", "sampling_rate"} / WAV path, URL, data
    URI or base64 (polyphase resampling for other rates)."""
    from ....preprocessing.media import load_audio

    return torch.from_numpy(load_audio(item, SAMPLE_RATE_IN))


def create_preprocessing_executor(model_path: str = "", overrides: dict | None = None, cache_keys: bool = True):
    """``cache_keys``: attach content keys of the request's audio and of its images + videos
    (``preprocessing.cache_key``), so the encoder stages reuse outputs of media they encoded
    before."""
    from ....preprocessing.cache_key import media_cache_key

    tok = load_tokenizer(model_path)
    n_window = 50

    def audio_tokens(n_samples: int) -> int:
        from ..audio_encoder import cnn_out_len

        frames = n_samples // 160
        cs = 2 * n_window
        full, rem = divmod(frames, cs)
        return full * cnn_out_len(cs) + (cnn_out_len(rem) if rem else 0)

    from ....preprocessing.vision_grid import resize_grid

    vcfg = loader.vision_config(model_path, overrides)
    unit = vcfg.patch_size * vcfg.spatial_merge_size

    def preprocess(payload: StagePayload) -> StagePayload:
        trace.mark(payload.request_id, "0_preprocess_start")
        inp = payload.request.inputs if isinstance(payload.request.inputs, dict) else {}
        raw_audios, raw_visual = list(inp.get("audios") or []), list(inp.get("images") or [])
        n_raw_images = len(raw_visual)
        raw_visual += list(inp.get("videos") or [])
        waves = [_load_audio(a) for a in (inp.get("audios") or [])]
        counts = [audio_tokens(w.numel()) for w in waves]
        images = [_load_image(im) for im in (inp.get("images") or [])]
        grids = []
        for im in images:
            th, tw = resize_grid(im.shape[0], im.shape[1], unit, vcfg.min_pixels, vcfg.max_pixels)
            grids.append((1, th // unit, tw // unit))
        from ....preprocessing.media import load_video, video_grid

        if (payload.request.params or {}).get("use_audio_in_video"):
            raise ValueError("use_audio_in_video is not supported: pass the video's audio track in 'audios'")
        videos = [load_video(v) for v in (inp.get("videos") or [])]
        vgrids = [video_grid(v["frames"], unit, vcfg.video_max_pixels, vcfg.video_min_pixels) for v in videos]
        if inp.get("prompt_token_ids") is not None and not waves and not images and not videos:
            ids = list(inp["prompt_token_ids"])
            p = torch.arange(len(ids), dtype=torch.int32)
            pos, delta, spans = torch.stack([p, p, p]), 0, []
            image_spans = []
        else:
            lay = build_prompt(tok, inp.get("messages"), inp.get("prompt"), counts, image_grids=grids,
                               video_grids=vgrids, video_second_per_grid=[v["second_per_grid"] for v in videos])
            ids = lay.ids
            pos, delta = mrope_positions(lay)
            spans = lay.audio_spans
            # images then videos: the vision stage encodes the items in this order
            image_spans = lay.image_spans + lay.video_spans
            images = images + videos
        data = {"prompt_token_ids": ids, "audio_waveforms": waves, "audio_spans": spans,
                "images": images, "image_spans": image_spans,
                "mrope_positions": pos, "mrope_delta": delta,
                "speech": _speech_requested(payload.request.params or {})}
        if cache_keys:
            data["audio_cache_key"] = media_cache_key("audio", raw_audios, sample_rate=16000, n_window=n_window)
            data["image_cache_key"] = media_cache_key("vision", raw_visual, unit=unit, images=n_raw_images)
        return StagePayload(payload.request_id, payload.request, data)

    return PreprocessingExecutor(preprocess)


# ----------------------------------------------------------------------------- encoders
def _device(device: str) -> str:
    """Reference configs say "cuda": this process's first visible GPU."""
    return "cuda:0" if device == "cuda" else device


def create_audio_encoder_executor(model_path: str = "", device: str = "cuda:0", max_batch_size: int = 32,
                                  overrides: dict | None = None, dtype=None, cache_size: int = 64):
    """``dtype``: accepted for reference configs; the tower runs in its configured dtype.
    ``cache_size``: outputs kept by the media key preprocessing attached (0: no cache)."""
    dev = torch.device(_device(device))
    enc = loader.get_audio_encoder(model_path, dev, overrides)
    mel = LogMel(enc.cfg.num_mel_bins, dev)

    def encode(inputs: dict) -> list:
        t0 = time.perf_counter()
        per_req = inputs["waves"]
        flat = [w for ws in per_req for w in ws]
        mels = mel.batch(flat) if flat else []
        if trace.ENABLED and dev.type == "cuda":
            torch.cuda.current_stream().synchronize()
            trace.batch("audio_mel", len(flat), time.perf_counter() - t0)
        outs = enc(mels) if mels else []
        if trace.ENABLED and dev.type == "cuda":
            torch.cuda.current_stream().synchronize()
            trace.batch("audio_encode_total", len(flat), time.perf_counter() - t0)
        res, i = [], 0
        for ws in per_req:
            res.append({"audio_embeds": outs[i:i + len(ws)]})
            i += len(ws)
        return res

    engine = create_encoder_engine(encode, max_batch_size=max_batch_size, device=dev, cache_size=cache_size,
                                   explicit_keys=True)

    def request_builder(payload: StagePayload):
        trace.mark(payload.request_id, "0b_audio_encoder_queued")
        waves = (payload.data or {}).get("audio_waveforms") or []
        return EncoderRequestData(inputs={"waves": waves}, skip=not waves,
                                  cache_key=(payload.data or {}).get("audio_cache_key") if waves else None)

    def result_builder(payload: StagePayload, out):
        if not isinstance(out, dict):  # skipped request (no audio)
            out = {"audio_embeds": None}
        trace.mark(payload.request_id, "1_audio_encoded")
        return StagePayload(payload.request_id, payload.request, out)

    return EngineExecutor(engine, request_builder, result_builder)


def create_image_encoder_executor(model_path: str = "", device: str = "cuda:0", max_batch_size: int = 32,
                                  overrides: dict | None = None, dtype=None, cache_size: int = 64):
    """The vision tower over a gathered burst of requests: one forward for every image of
    the batch (ragged attention keeps images apart), split back per request.  ``cache_size``:
    outputs kept by the media key preprocessing attached (0: no cache)."""
    from ..vision_encoder import encode_images

    dev = torch.device(_device(device))
    # built now, not on the first request: building ends with a device-wide synchronize, which
    # must not run while another stage's engine thread is capturing its CUDA graphs
    loader.get_vision_encoder(model_path, dev, overrides)

    def encode(inputs: dict) -> list:
        per_req = inputs["images"]
        flat = [im for ims in per_req for im in ims]
        t0 = time.perf_counter()
        out = encode_images(model_path, dev, flat, overrides) if flat else None
        if trace.ENABLED and flat:
            if dev.type == "cuda":   # this stream only: another stage may be capturing a graph
                torch.cuda.current_stream(dev).synchronize()
            trace.batch("image_encode", len(flat), time.perf_counter() - t0)
        res, i = [], 0
        for ims in per_req:
            n = len(ims)
            res.append({"image_embeds": out["image_embeds"][i:i + n],
                        "deepstack": [d[i:i + n] for d in out["deepstack"]],
                        "image_grids": out["image_grids"][i:i + n]})
            i += n
        return res

    engine = create_encoder_engine(encode, max_batch_size=max_batch_size, device=dev, cache_size=cache_size,
                                   explicit_keys=True)

    def request_builder(payload: StagePayload):
        images = (payload.data or {}).get("images") or []
        if images:
            trace.mark(payload.request_id, "0c_image_encoder_queued")
        return EncoderRequestData(inputs={"images": images}, skip=not images,
                                  cache_key=(payload.data or {}).get("image_cache_key") if images else None)

    def result_builder(payload: StagePayload, out):
        if not isinstance(out, dict):  # skipped request (no image)
            out = {"image_embeds": None}
        else:
            trace.mark(payload.request_id, "1c_image_encoded")
        return StagePayload(payload.request_id, payload.request, out)

    return EngineExecutor(engine, request_builder, result_builder)


def create_aggregate_executor(**_):
    return PreprocessingExecutor(lambda p: p)


# ----------------------------------------------------------------------------- thinker
def create_thinker_executor(model_path: str = "", device: str = "cuda:0", max_batch: int = 64,
                            max_context: int = 4096, max_prefill_tokens: int = 8192, speech_target: str | None = None,
                            accept_hidden_layer: int = 24, overrides: dict | None = None, use_graphs: bool = True,
                            model=None, tokenizer=None, eos_token_ids=THINKER_EOS_IDS, prefix_cache: bool = True,
                            tp_size: int = 1, ep_size: int = 1, gpus: list | None = None):
    """The thinker stage over the paged engine; ``model`` / ``tokenizer`` / ``eos_token_ids``
    let another omni model (same request layout: prompt ids + audio / image spans) reuse it.

    ``tp_size`` / ``ep_size`` > 1 serve the thinker with a rank group of that many GPUs
    (``gpus``: logical GPU per rank, default this device and the next ones): tensor
    parallel (every rank runs every request) or expert parallel with data-parallel
    attention (each request on one rank, the experts sharded)."""
    dev = torch.device(device)
    pages = max_batch * ((max_context + 63) // 64) + 8
    engine_args = dict(max_batch=max_batch, max_prefill_tokens=max_prefill_tokens, max_context=max_context,
                       use_graphs=use_graphs and dev.type == "cuda", eos_token_ids=tuple(eos_token_ids),
                       prefix_cache=prefix_cache)
    if tp_size > 1 or ep_size > 1:
        from ....parallel.rank_group import GroupedAREngine, GroupSpec, StageRankGroup

        if tp_size > 1 and ep_size > 1:
            # attention TP inside data-parallel groups of tp_size ranks, experts over ep_size ranks
            if ep_size % tp_size != 0:
                raise ValueError(f"ep_size {ep_size} must be a multiple of tp_size {tp_size}")
            mode, world, group_tp = "ep", ep_size, tp_size
        else:
            mode, world = ("tp", tp_size) if tp_size > 1 else ("ep", ep_size)
            group_tp = 1
        if mode == "ep" and speech_target is not None:
            raise NotImplementedError("expert-parallel thinker groups serve text output; the talker needs the "
                                      "hidden states of every request on the leader (use tp_size)")
        if dev.type == "cuda":
            torch.cuda.set_device(dev)
        base = dev.index if dev.index is not None else 0
        spec = GroupSpec(mode=mode, world=world, gpus=list(gpus) if gpus else list(range(base, base + world)),
                         builder="sglang_omni_b200.models.qwen3_omni.loader.build_thinker_rank",
                         builder_args={"model_path": model_path, "overrides": overrides,
                                       "max_tokens": max(max_prefill_tokens, max_batch)},
                         engine_args=engine_args, kv_pages=pages, tp=group_tp)
        rg = StageRankGroup(spec)
        engine = rg.start()
        model = rg.model
        adapter = PagedAREngineAdapter(engine, threaded=GroupedAREngine(engine, rg))
    else:
        model = model if model is not None else loader.get_thinker(model_path, dev, overrides)
        cfg = model.cfg
        pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, pages, dev, cfg.dtype)
        engine = AREngine(model, pool, **engine_args)
        adapter = PagedAREngineAdapter(engine)
    tok = tokenizer if tokenizer is not None else load_tokenizer(model_path, model.cfg.vocab_size)
    cfg = model.cfg
    detoks: dict[str, IncrementalDetokenizer] = {}
    accept = min(accept_hidden_layer, cfg.num_layers)

    ex = EngineExecutor(adapter, None, None, None)

    def request_builder(payload: StagePayload) -> ARRequest:
        d = payload.data
        trace.mark(payload.request_id, "1b_thinker_queued")
        sp = sampling_for(payload, "thinker")
        ids = list(d["prompt_token_ids"])
        req = ARRequest(rid=payload.request_id, prompt_ids=ids, sampling=sp,
                        max_new_tokens=sp.max_new_tokens or 256)
        req.mrope_positions = d.get("mrope_positions")
        req.mrope_delta = int(d.get("mrope_delta") or 0)
        aud = d.get("audio_embeds") or []
        spans = d.get("audio_spans") or []
        img = d.get("image_embeds") or []
        img_spans = d.get("image_spans") or []
        if aud or img:
            mm_index = torch.full((len(ids),), -1, dtype=torch.int32)
            base, mats = 0, []
            for (a, b), emb in list(zip(spans, aud)) + list(zip(img_spans, img)):
                n = min(b - a, emb.shape[0])
                mm_index[a:a + n] = torch.arange(base, base + n, dtype=torch.int32)
                base += emb.shape[0]
                mats.append(emb)
            req.mm_index = mm_index
            req.mm_embeds = torch.cat(mats, 0)
        ds = d.get("deepstack")
        if ds and img_spans:
            pos = torch.cat([torch.arange(a, b) for a, b in img_spans])
            req.deepstack = [torch.cat(list(layer), 0) for layer in ds]
            req.ds_positions = pos
        speech = bool(d.get("speech")) and speech_target is not None
        if speech:
            req.capture_prompt_layer = accept if aud else None
            sent = {"first": True}

            def on_token(r, token, info, _rid=payload.request_id, _sent=sent, _spans=spans):
                msg = {"token_id": int(token)}
                if _sent["first"]:
                    _sent["first"] = False
                    ph = r.extra.get("prompt_hidden")
                    if ph:
                        # the prefill rows are complete (this runs after the first token's event);
                        # the talker gathers the multimodal rows on its own stream
                        n = sum(t.shape[0] for t in ph)
                        mask = torch.zeros(n, dtype=torch.bool)
                        for a, b in _spans:
                            mask[a:b] = True
                        msg["mm_mask"] = mask
                        msg["mm_hidden_parts"] = list(ph)
                lane = fastlane.get(speech_target)
                if lane is not None:      # talker in this process: straight to its thread
                    lane.deliver_many([(_rid, msg)])
                elif ex._stream_fn is not None:
                    ex._stream_fn(_rid, msg, speech_target)

            req.on_token = on_token
        detoks[payload.request_id] = IncrementalDetokenizer(tok)
        return req

    def stream_builder(payload: StagePayload, chunk):
        token, _ = chunk
        trace.mark(payload.request_id, "2_thinker_first_token")
        d = detoks.get(payload.request_id)
        text = d.push(token) if d is not None else ""
        return {"modality": "text", "token_ids": [int(token)], "text": text}

    def result_builder(payload: StagePayload, r: ARRequest) -> StagePayload:
        detoks.pop(payload.request_id, None)
        text = tok.decode(r.output_ids, skip_special_tokens=True)
        data = {"token_ids": list(r.output_ids), "text": text, "finish_reason": r.finish_reason,
                "usage": {"prompt_tokens": len(r.prompt_ids), "completion_tokens": len(r.output_ids),
                          "total_tokens": len(r.prompt_ids) + len(r.output_ids)},
                "ttft_s": (r.first_token_time - r.arrival) if r.first_token_time else None}
        return StagePayload(payload.request_id, payload.request, data)

    ex.request_builder = request_builder
    ex.stream_builder = stream_builder
    ex.result_builder = result_builder
    ex.ar_engine = engine
    return ex


def create_sglang_thinker_executor_from_config(model_path: str = "", device: str = "cuda",
                                               thinker_max_seq_len: int = 8192, speech_enabled: bool = False,
                                               **kw):
    """Factory name and arguments of the reference's thinker stage
    (sglang_omni/models/qwen3_omni/config.py:160-168): the paged-engine thinker, streaming
    to the talker when speech is enabled."""
    from .next_stage import TALKER_AR_STAGE

    kw.setdefault("max_context", thinker_max_seq_len)
    return create_thinker_executor(model_path=model_path, device=_device(device),
                                   speech_target=TALKER_AR_STAGE if speech_enabled else None, **kw)


def create_talker_ar_executor_from_config(model_path: str = "", device: str = "cuda", talker_max_seq_len: int = 8192,
                                          speech_enabled: bool = True, feedback_enabled: bool = True, **kw):
    """Factory name and arguments of the reference's talker stage (config.py:179-192).  The
    code predictor runs inside this stage (one CUDA graph per frame); its frames go to the
    ``code_predictor`` stage of the reference layout, which forwards them to code2wav."""
    from .next_stage import CODE_PREDICTOR_STAGE

    kw.setdefault("max_frames", talker_max_seq_len)
    return TalkerStreamingExecutor(model_path, _device(device), code_target=CODE_PREDICTOR_STAGE, **kw)


def create_decode_executor(**_):
    def run(payload: StagePayload) -> StagePayload:
        d = dict(payload.data or {})
        meta = payload.request.metadata or {}
        if "usage" in d and meta.get("engine_time_s") is not None:
            d["usage"] = dict(d["usage"], engine_time_s=meta["engine_time_s"])
        return StagePayload(payload.request_id, payload.request, d)

    return PreprocessingExecutor(run)


# ----------------------------------------------------------------------------- talker (+ code predictor)
class TalkerStreamingExecutor(ResultQueueMixin, Executor):
    """Runs the SpeechGenerator on its own thread; inbound thinker tokens come
    through the stage mailbox, code frames go to ``code_target``."""

    def __init__(self, model_path: str, device: str, max_streams: int = 64, code_target: str = "code2wav",
                 overrides: dict | None = None, max_frames: int = 4096, use_graphs: bool = True,
                 tail_frames: int = 50, stage_name: str = "talker_ar"):
        super().__init__()
        self.stage_name = stage_name
        dev = torch.device(device)
        self.device = dev
        self.talker = loader.get_talker(model_path, dev, overrides)
        self.embed = loader.thinker_embedding(model_path, dev, overrides)
        self.gen = SpeechGenerator(self.talker, self.embed, max_streams=max_streams,
                                   use_graphs=use_graphs and dev.type == "cuda", tail_frames=tail_frames)
        self.code_target = code_target
        self.max_frames = max_frames
        self._cv = threading.Condition()
        self._new: deque = deque()        # (rid, prompt_ids, speaker)
        self._tokens: dict[str, list] = {}
        self._first: dict[str, dict] = {}
        self._done: set[str] = set()
        self._aborted: set[str] = set()
        self._pending: dict[str, dict] = {}
        self._thread: threading.Thread | None = None
        self._loop: asyncio.AbstractEventLoop | None = None
        self._stop = False
        self.error: BaseException | None = None

    async def start(self):
        self._loop = asyncio.get_running_loop()
        fastlane.register(self.stage_name, self)
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name="talker", daemon=True)
            self._thread.start()

    async def stop(self):
        fastlane.unregister(self.stage_name, self)
        with self._cv:
            self._stop = True
            self._cv.notify_all()

    def deliver_many(self, items):
        """Fast lane from the thinker's engine thread: token (and first-token prompt hidden
        state) items of any streams, applied under the generator's lock."""
        with self._cv:
            for rid, data in items:
                if "mm_hidden_parts" in data:
                    self._first[rid] = {"mm_mask": data["mm_mask"], "parts": data["mm_hidden_parts"]}
                self._tokens.setdefault(rid, []).append(int(data["token_id"]))
            self._cv.notify_all()

    async def add_request(self, payload: StagePayload) -> None:
        rid = payload.request_id
        d = payload.data or {}
        meta = payload.request.metadata or {}
        speaker = (meta.get("audio") or {}).get("voice") or meta.get("voice")
        self._pending[rid] = {"payload": payload, "t0": time.perf_counter()}
        with self._cv:
            self._tokens.setdefault(rid, [])      # fast-lane tokens may have arrived already
            self._new.append((rid, list(d.get("prompt_token_ids") or []), speaker))
            self._cv.notify_all()
        asyncio.ensure_future(self._pump(rid))

    async def _pump(self, rid: str):
        """Moves thinker chunks from the mailbox to the generator thread."""
        try:
            while True:
                item = await self._mailbox.get(rid)
                if item is None:
                    break
                with self._cv:
                    data = item.data
                    if "mm_hidden_parts" in data:
                        self._first[rid] = {"mm_mask": data["mm_mask"], "parts": data["mm_hidden_parts"]}
                    self._tokens.setdefault(rid, []).append(int(data["token_id"]))
                    self._cv.notify_all()
        except Exception as exc:  # thinker stream error
            self._finish(rid, error=str(exc))
            return
        with self._cv:
            self._done.add(rid)
            self._cv.notify_all()

    def _finish(self, rid: str, error: str | None = None, frames: int = 0):
        info = self._pending.pop(rid, None)
        if info is None:
            return
        p = info["payload"]
        if error is not None:
            item = StageError(rid, error)
        else:
            item = StagePayload(rid, p.request, {"num_frames": frames})
        self._loop.call_soon_threadsafe(self._results().put_nowait, item)

    async def abort(self, request_id: str) -> None:
        with self._cv:
            self._aborted.add(request_id)
            self._cv.notify_all()

    # ---------------------------------------------------------------- generator thread
    def _run(self):
        stream = own_stream(self.device)
        if stream is not None:
            torch.cuda.set_stream(stream)  # frames wait only for talker work, not for queued thinker steps
        try:
            with torch.inference_mode():
                self.gen.capture_all()
                self._loop_body()
        except BaseException as exc:
            log.exception("talker thread failed")
            self.error = exc
            for rid in list(self._pending):
                self._finish(rid, error=f"talker failed: {exc}")

    def _emit(self, streams, codes: torch.Tensor):
        host = codes.cpu().tolist()
        eos = self.talker.special.codec_eos
        lane = fastlane.get(self.code_target)   # vocoder in this process: one hand-off per step
        batch = []
        for s, c in zip(streams, host):
            if c[0] == eos or s.frames >= s.max_frames:
                s.finished = True
                if lane is None:
                    self._stream_fn(s.rid, {"codes": [], "eos": True}, self.code_target)
                self._finish(s.rid, frames=s.frames)
                self.gen.remove(s.rid)
            else:
                trace.mark(s.rid, "3_talker_first_frame")
                if trace.ENABLED and s.frames >= 4:
                    trace.mark(s.rid, "3b_talker_frame_4")
                if lane is not None:
                    batch.append((s.rid, {"codes": c}))
                else:
                    self._stream_fn(s.rid, {"codes": c}, self.code_target)
        if batch:
            lane.deliver_many(batch)

    def _loop_body(self):
        gen = self.gen
        while True:
            with self._cv:
                while not self._stop and not self._has_work():
                    self._cv.wait(timeout=0.5)
                if self._stop:
                    return
                aborted, self._aborted = self._aborted, set()
                new_ready = []
                keep = deque()
                while self._new:
                    rid, ids, spk = self._new.popleft()
                    if rid in aborted:
                        continue
                    if self._tokens.get(rid):
                        new_ready.append((rid, ids, spk, self._tokens[rid][:1], self._first.pop(rid, None)))
                        self._tokens[rid] = self._tokens[rid][1:]
                    else:
                        keep.append((rid, ids, spk))
                self._new = keep
                pending_tokens = {rid: self._tokens[rid] for rid in list(self._tokens) if self._tokens[rid]
                                  and rid in gen.streams}
                for rid in pending_tokens:
                    self._tokens[rid] = []
                done = {rid for rid in self._done if rid in gen.streams}
                self._done -= done
            for rid in aborted:
                if rid in gen.streams:
                    gen.remove(rid)
                self._pending.pop(rid, None)
            # new streams: build the HF-parity prefill and run it batched
            new_streams = []
            for rid, ids, spk, first, mm in new_ready:
                pre, trail, pad_e, eos_e = build_talker_prefill(
                    self.talker, self.embed, ids, first, None if mm is None else mm["mm_mask"][:len(ids)],
                    None if mm is None else self._scatter_mm(mm, len(ids)), spk)
                done_now = rid in self._done
                new_streams.append(gen.add_stream(rid, pre, trail, pad_e, eos_e, thinker_done=done_now,
                                                  max_frames=self.max_frames))
            if new_streams:
                self._emit(new_streams, gen.prefill(new_streams))
            # trailing text from newly arrived thinker tokens (one batched projection)
            if pending_tokens:
                rids = list(pending_tokens)
                flat = [t for r in rids for t in pending_tokens[r]]
                proj = self.talker.project_text(self.embed[h2d(flat, self.device, torch.long)])
                o = 0
                for r in rids:
                    n = len(pending_tokens[r])
                    gen.push_trailing(r, proj[o:o + n], done=False)
                    o += n
            for rid in done:
                gen.push_trailing(rid, None, done=True)
            ready = [s for s in gen.ready_streams() if len(self._pending) and s.rid in self._pending]
            if ready:
                self._emit(ready, gen.step(ready))

    def _scatter_mm(self, mm, L):
        parts = [adopt(t) for t in mm["parts"]]          # produced on the thinker's stream
        hid = torch.cat(parts, 0) if len(parts) > 1 else parts[0]
        full = torch.zeros(L, hid.shape[-1], dtype=hid.dtype, device=self.device)
        mask = mm["mm_mask"][:L]
        sel = (mask.cpu() if mask.is_cuda else mask).nonzero().view(-1)   # host-side: no device sync
        if sel.numel():
            full.index_copy_(0, h2d(sel, self.device), hid.to(self.device).index_select(0, h2d(sel, hid.device)))
        return full

    def _has_work(self) -> bool:
        if self._aborted or self._done:
            return True
        if any(self._tokens.get(rid) for rid, *_ in self._new):
            return True
        if any(self._tokens.get(rid) for rid in self.gen.streams):
            return True
        return bool(self.gen.ready_streams())


def create_talker_executor(model_path: str = "", device: str = "cuda:0", max_streams: int = 64,
                           overrides: dict | None = None, use_graphs: bool = True, tail_frames: int = 50,
                           max_frames: int = 4096):
    return TalkerStreamingExecutor(model_path, device, max_streams, overrides=overrides, use_graphs=use_graphs,
                                   tail_frames=tail_frames, max_frames=max_frames)


# ----------------------------------------------------------------------------- code2wav
class Code2WavStreamingExecutor(ResultQueueMixin, Executor):
    """Incremental vocoding of every active stream; emits float32 PCM chunks
    (12.5 Hz frames -> 24 kHz) to the client as they are produced.

    One decoder loop serves all streams: whenever frames arrive it decodes every
    stream that has a chunk ready in one batched forward per step shape
    (instead of one forward per stream), off the event loop.

    ``mode``: "stateful" (default) keeps each stream's transformer keys / values
    and convolution history, so a chunk runs only its new frames and the stream's
    chunks add up to the full-sequence waveform (``code2wav_stateful``), for up to
    ``max_open_streams`` concurrent streams; "window" re-runs ``left_context``
    frames before every chunk, as the reference executor does.  ``max_streams``:
    largest batch captured as one CUDA graph."""

    def __init__(self, model_path: str, device: str, chunk: int = 10, left_context: int = 25,
                 first_chunk: int | None = None, overrides: dict | None = None, use_graphs: bool = True,
                 max_streams: int = 32, mode: str = "stateful", max_open_streams: int = 128,
                 max_frames: int = 16384):
        super().__init__()
        dev = torch.device(device)
        self.model = loader.get_code2wav(model_path, dev, overrides)
        if mode == "stateful":
            self.sc = StatefulStreamingCode2Wav(self.model, chunk, first_chunk, max(max_open_streams, max_streams),
                                                max_frames, use_graphs=use_graphs)
            if self.sc.graphs is not None:
                self.sc.graphs.max_batch = max_streams
        elif mode == "window":
            graphs = Code2WavGraphs(self.model, max_streams) if use_graphs and dev.type == "cuda" else None
            self.sc = StreamingCode2Wav(self.model, chunk, left_context, first_chunk, graphs=graphs)
        else:
            raise ValueError(f"code2wav mode {mode!r}: expected 'stateful' or 'window'")
        # its own high-priority stream: a chunk's kernels and its host copy wait for nothing
        # the thinker / talker threads queued
        self._stream = torch.cuda.Stream(device=dev, priority=-1) if dev.type == "cuda" else None
        self._streams: dict[str, asyncio.Queue] = {}
        self._audio: dict[str, list] = {}
        self._finals: set[str] = set()
        self._flushed: dict[str, asyncio.Future] = {}
        self._wake: asyncio.Event | None = None
        self._loop_task: asyncio.Task | None = None
        self.stage_name = "code2wav"
        self._lane_lock = threading.Lock()
        self._lane_items: list = []      # fast-lane frames not yet applied on the event loop
        self._early: dict[str, list] = {}  # frames of streams whose request has not arrived yet
        self._loop: asyncio.AbstractEventLoop | None = None

    async def start(self):
        self._loop = asyncio.get_running_loop()
        if self.sc.graphs is not None:
            await asyncio.to_thread(self._capture)
        fastlane.register(self.stage_name, self)

    def _capture(self):
        with torch.cuda.stream(self._stream), torch.inference_mode():
            self.sc.capture_graphs()

    def _decode(self, ready, finals):
        """One batched decode of the ready streams on this stage's stream; host arrays."""
        if self._stream is None:
            return self.sc.decode_ready(ready, False, finals, to_host=True)
        with torch.cuda.stream(self._stream), torch.inference_mode():
            return self.sc.decode_ready(ready, False, finals, to_host=True)

    async def stop(self):
        fastlane.unregister(self.stage_name, self)

    def deliver_many(self, items):
        """Fast lane from the talker thread: one callback on the event loop per batch."""
        with self._lane_lock:
            first = not self._lane_items
            self._lane_items.extend(items)
        if first and self._loop is not None:
            self._loop.call_soon_threadsafe(self._apply_lane)

    def _apply_lane(self):
        with self._lane_lock:
            items, self._lane_items = self._lane_items, []
        woke = False
        for rid, data in items:
            if rid not in self._streams:
                if len(self._early) < 4096:   # frames of a stream that ended or was aborted are dropped
                    self._early.setdefault(rid, []).append(data)
                continue
            self.sc.add_codes(rid, torch.tensor(data["codes"], dtype=torch.long))
            ready = self.sc.ready(rid)
            if ready:
                trace.mark(rid, "3c_vocoder_chunk_ready")
            woke = woke or ready
        if woke and self._wake is not None:
            self._wake.set()

    async def add_request(self, payload: StagePayload) -> None:
        rid = payload.request_id
        if self._wake is None:
            self._wake = asyncio.Event()
        if self._loop is None:
            self._loop = asyncio.get_running_loop()
        if self._loop_task is None or self._loop_task.done():
            self._loop_task = asyncio.ensure_future(self._decoder_loop())
        self._streams[rid] = asyncio.Queue()
        self._audio[rid] = []
        self._flushed[rid] = asyncio.get_running_loop().create_future()
        for data in self._early.pop(rid, []):
            self.sc.add_codes(rid, torch.tensor(data["codes"], dtype=torch.long))
        if self.sc.ready(rid):
            self._wake.set()
        asyncio.ensure_future(self._run(payload))

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

    async def _decoder_loop(self):
        while True:
            await self._wake.wait()
            self._wake.clear()
            live = [r for r in self._streams if r in self.sc.streams]
            finals = {r for r in live if r in self._finals}
            ready = [r for r in live if self.sc.ready(r, r in finals)]
            if ready:
                for r in ready:
                    trace.mark(r, "3d_vocoder_decode_start")
                try:
                    out = await asyncio.to_thread(self._decode, ready, finals)
                except Exception as exc:  # fail the streams of this batch only
                    log.exception("code2wav batch failed")
                    for r in ready:
                        f = self._flushed.get(r)
                        if f is not None and not f.done():
                            f.set_exception(exc)
                    continue
                now = time.perf_counter()
                for r, a in out.items():
                    trace.mark(r, "4_first_audio_chunk")
                    if r in self._audio:
                        self._audio[r].append(a)
                    q = self._streams.get(r)
                    if q is not None:
                        q.put_nowait({"modality": "audio", "audio_waveform": a, "sample_rate": SAMPLE_RATE_OUT,
                                      "t": now})
            for r in finals:
                if not self.sc.ready(r, True):
                    f = self._flushed.get(r)
                    if f is not None and not f.done():
                        f.set_result(True)
            if any(self.sc.ready(r, r in self._finals) for r in self._streams if r in self.sc.streams):
                self._wake.set()

    async def _run(self, payload: StagePayload):
        rid = payload.request_id
        try:
            while True:
                item = await self._mailbox.get(rid)
                if item is None or item.data.get("eos"):
                    break
                self.sc.add_codes(rid, torch.tensor(item.data["codes"], dtype=torch.long))
                if self.sc.ready(rid):
                    self._wake.set()
            if rid not in self.sc.streams:  # no frame at all
                self.sc.add_codes(rid, torch.zeros(0, self.model.cfg.num_quantizers, dtype=torch.long))
            self._finals.add(rid)
            self._wake.set()
            await self._flushed[rid]
            audio = np.concatenate(self._audio.pop(rid)) if self._audio.get(rid) else np.zeros(0, np.float32)
            self._results().put_nowait(StagePayload(rid, payload.request,
                                                    {"audio_waveform": audio, "sample_rate": SAMPLE_RATE_OUT}))
        except asyncio.CancelledError:
            raise
        except Exception as exc:
            self._results().put_nowait(StageError(rid, f"code2wav: {exc}"))
        finally:
            self._cleanup(rid)

    def _cleanup(self, rid: str):
        self.sc.close(rid)
        self._early.pop(rid, None)
        self._finals.discard(rid)
        self._flushed.pop(rid, None)
        self._audio.pop(rid, None)
        q = self._streams.pop(rid, None)
        if q is not None:
            q.put_nowait(None)

    async def abort(self, request_id: str) -> None:
        f = self._flushed.get(request_id)
        if f is not None and not f.done():
            f.cancel()
        self._cleanup(request_id)


def create_code2wav_executor(model_path: str = "", device: str = "cuda:0", chunk: int = 10,
                             left_context: int = 25, first_chunk: int | None = None, overrides: dict | None = None,
                             use_graphs: bool = True, max_streams: int = 32, mode: str = "stateful",
                             max_open_streams: int = 128, max_frames: int = 16384):
    return Code2WavStreamingExecutor(model_path, device, chunk, left_context, first_chunk, overrides,
                                     use_graphs=use_graphs, max_streams=max_streams, mode=mode,
                                     max_open_streams=max_open_streams, max_frames=max_frames)
