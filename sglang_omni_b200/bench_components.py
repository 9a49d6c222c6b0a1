"""Component timings against the reference's own stage code, on one GPU.

    python -m sglang_omni_b200.bench_components [--ref-path baseline/_ref]

The reference's thinker and talker need ``sglang`` (not in this image), but its
audio-tower, vision-tower and Code2Wav stage components run on transformers alone.  This
script writes one random-weight checkpoint (a Qwen3-Omni ``config.json`` with
the published architecture and ``thinker.audio_tower.*`` / ``thinker.visual.*`` /
``code2wav.*`` tensors in safetensors) that both implementations load through their own loaders, then
times each on the same inputs with CUDA events (after warm-up, L2 flushed):

* audio tower, speech-input shape: 32 streams of 10 s (1000 log-mel frames), one
  batched forward.  Reference: ``Qwen3OmniAudioEncoder.forward``
  (sglang_omni/models/qwen3_omni/components/audio_encoder.py:58-90);
* vision tower, image+text shape: 64 images of 448 x 448 (196 merged
  tokens each), one batched forward.  Reference:
  ``Qwen3OmniImageEncoder.forward`` (sglang_omni/models/qwen3_omni/components/
  image_encoder.py:131-180, HF vision encoder with its Linear patch embed);
* Code2Wav streaming chunk, 32 streams x (25 context + 10 new frames).
  Reference: ``_decode_incremental`` per stream under its GPU lock, i.e. one
  model call per stream (code2wav_executor.py:190-232); ours: one batched
  call of ``StreamingCode2Wav`` over the 32 streams.

It prints one JSON line per component with both times and the relative
difference of the outputs.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import types

import numpy as np
import torch


def _time(fn, iters=10, flush=None):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        tot += a.elapsed_time(b)
    return tot / iters


class _Placeholder(types.ModuleType):
    """Stands in for a file-decoding library the image lacks; any attribute is another
    placeholder, so ``from lib import name`` succeeds and only a call would fail."""

    def __getattr__(self, attr):
        if attr.startswith("__"):
            raise AttributeError(attr)
        sub = _Placeholder(f"{self.__name__}.{attr}")
        setattr(self, attr, sub)
        return sub

    def __call__(self, *a, **k):
        raise RuntimeError(f"{self.__name__} is not installed")


def _import_reference(path: str) -> None:
    """Import the reference's vision-encoder and Code2Wav components from `path`.  Its
    package __init__ pulls in its media decoders, whose libraries (PyAV, librosa,
    qwen_vl_utils, ...) are not in this image; the timed components never call them, so
    placeholder modules stand in for whichever of them is missing."""
    import importlib.machinery

    import transformers  # noqa: F401  (its package probes run before any placeholder exists)

    sys.path.insert(0, path)
    for _ in range(16):
        try:
            import sglang_omni.models.qwen3_omni.components.audio_encoder  # noqa: F401
            import sglang_omni.models.qwen3_omni.components.code2wav_executor  # noqa: F401
            import sglang_omni.models.qwen3_omni.components.image_encoder  # noqa: F401
            return
        except ModuleNotFoundError as exc:
            name = (exc.name or "").split(".")[0]
            if not name or name.startswith("sglang_omni") or name in sys.modules:
                raise
            mod = _Placeholder(name)
            mod.__spec__ = importlib.machinery.ModuleSpec(name, None)
            mod.__path__ = []
            sys.modules[name] = mod
            for k in [k for k in sys.modules if k.startswith("sglang_omni")]:
                del sys.modules[k]
    raise ImportError("the reference's components did not import")


def _write_checkpoint(path: str, dev) -> None:
    """config.json of the published architecture + random thinker.visual / code2wav tensors."""
    from safetensors.torch import save_file
    from transformers.models.qwen3_omni_moe import configuration_qwen3_omni_moe as hc
    from transformers.models.qwen3_omni_moe import modeling_qwen3_omni_moe as hm

    cfg = hc.Qwen3OmniMoeConfig()
    # the published checkpoint's vision merger projects to the thinker width (2048)
    cfg.thinker_config.vision_config.out_hidden_size = cfg.thinker_config.text_config.hidden_size
    # ... and its audio tower uses 50-frame windows and the same output width
    cfg.thinker_config.audio_config.n_window = 50
    cfg.thinker_config.audio_config.output_dim = cfg.thinker_config.text_config.hidden_size
    cfg.save_pretrained(path)
    torch.manual_seed(0)
    tensors = {}
    aud = hm.Qwen3OmniMoeAudioEncoder(cfg.thinker_config.audio_config).to(dev, torch.bfloat16)
    for k, v in aud.state_dict().items():
        tensors["thinker.audio_tower." + k] = (v.float().normal_(0, 0.02) if v.dim() > 1 else v.float()).bfloat16().cpu()
    del aud
    vis = hm.Qwen3OmniMoeVisionEncoder(cfg.thinker_config.vision_config).to(dev, torch.bfloat16)
    for k, v in vis.state_dict().items():
        tensors["thinker.visual." + k] = (v.float().normal_(0, 0.02) if v.dim() > 1 else v.float()).bfloat16().cpu()
    del vis
    c2w = hm.Qwen3OmniMoeCode2Wav(cfg.code2wav_config).to(dev, torch.bfloat16)
    for k, v in c2w.state_dict().items():
        tensors["code2wav." + k] = (v.float().normal_(0, 0.02) if v.dim() > 1 else v.float()).bfloat16().cpu()
    del c2w
    save_file(tensors, os.path.join(path, "model.safetensors"))


def audio(ckpt: str, dev, flush, n_streams: int = 32) -> dict:
    from sglang_omni.models.qwen3_omni.components.audio_encoder import Qwen3OmniAudioEncoder

    from .models.qwen3_omni import loader

    ref = Qwen3OmniAudioEncoder(ckpt, device=str(dev), dtype="bfloat16")
    ours = loader.get_audio_encoder(ckpt, dev)
    g = torch.Generator().manual_seed(2)
    mels = [torch.randn(128, 1000, generator=g) for _ in range(n_streams)]   # 10 s of 100 Hz log-mel each
    feats = torch.cat(mels, 1).to(dev)
    lens = torch.full((n_streams,), 1000, dtype=torch.long, device=dev)
    mels_d = [m.to(dev) for m in mels]

    def ref_fwd():
        return ref(input_features=feats, audio_feature_lengths=lens)["audio_embeds"]

    with torch.no_grad():
        r = ref_fwd()
        o = torch.cat(ours(mels_d), 0)
        t_ref = _time(ref_fwd, flush=flush)
        t_ours = _time(lambda: ours(mels_d), flush=flush)
    err = float((o.float() - r.float()).norm() / r.float().norm())
    return {"component": f"audio tower, {n_streams} x 10 s (1000 mel frames each), one forward",
            "reference_ms": round(t_ref, 3), "ours_ms": round(t_ours, 3), "speedup": round(t_ref / t_ours, 2),
            "rel_diff": round(err, 4), "reference_call": "Qwen3OmniAudioEncoder.forward"}


def vision(ckpt: str, dev, flush, n_images: int = 64) -> dict:
    from sglang_omni.models.qwen3_omni.components.image_encoder import Qwen3OmniImageEncoder

    from .models.qwen3_omni import loader
    from .models.qwen3_omni.vision_encoder import image_to_patches

    ref = Qwen3OmniImageEncoder(ckpt, device=str(dev), dtype="bfloat16")
    ours = loader.get_vision_encoder(ckpt, dev)
    rng = np.random.default_rng(0)
    imgs = [rng.integers(0, 256, (448, 448, 3), dtype=np.uint8) for _ in range(n_images)]
    patches, grids = zip(*[image_to_patches(im, ours.cfg) for im in imgs])
    px = torch.cat(patches, 0).to(dev)
    grid_t = torch.tensor(grids, device=dev)
    note = "Qwen3OmniImageEncoder.forward"

    def ref_fwd():
        return ref(pixel_values=px, image_grid_thw=grid_t)["image_embeds"]

    with torch.no_grad():
        try:
            r = ref_fwd()
        except ValueError:
            # The component unpacks the vision module's output as (embeds, deepstack); the
            # installed transformers returns a 3-field output object instead, so the module
            # the component built (with its Linear patch embed) is called directly.
            note = "Qwen3OmniImageEncoder.visual (component forward fails on this transformers)"

            def ref_fwd():
                return ref.visual(px.to(ref.visual.dtype), grid_thw=grid_t).pooler_output

            r = ref_fwd()
        o, _ = ours(px, list(grids))
        t_ref = _time(ref_fwd, flush=flush)
        t_ours = _time(lambda: ours(px, list(grids)), flush=flush)
    err = float((o.float() - r.float()).norm() / r.float().norm())
    return {"component": f"vision tower, {n_images} x 448x448 images (196 tokens each), one forward",
            "reference_ms": round(t_ref, 3), "ours_ms": round(t_ours, 3), "speedup": round(t_ref / t_ours, 2),
            "rel_diff": round(err, 4), "reference_call": note}


def code2wav(ckpt: str, dev, flush, n_streams: int = 32) -> dict:
    from sglang_omni.models.qwen3_omni.components.code2wav_executor import load_code2wav_model

    from .models.qwen3_omni import loader
    from .models.qwen3_omni.code2wav import StreamingCode2Wav

    ref = load_code2wav_model(ckpt, device=str(dev), dtype="bfloat16")
    ours = loader.get_code2wav(ckpt, dev)
    S, ctx, new = n_streams, 25, 10
    Q = ours.cfg.num_quantizers
    g = torch.Generator().manual_seed(1)
    codes = torch.randint(0, ours.cfg.codebook_size, (S, Q, ctx + new), generator=g)
    up = ours.cfg.total_upsample

    def ref_chunks():
        outs = []
        for s in range(S):   # the reference decodes one stream at a time (GPU lock)
            wav = ref(codes[s:s + 1].to(dev))
            outs.append(wav[..., ctx * up:].reshape(-1))
        return outs

    sc = StreamingCode2Wav(ours, chunk=new, left_context=ctx, first_chunk=new)

    def ours_chunks():
        for s in range(S):
            sc.close(f"s{s}")
            sc.add_codes(f"s{s}", codes[s].t())
            st = sc.streams[f"s{s}"]
            st.emitted_frames = ctx          # the context frames were emitted by earlier chunks
        return sc.decode_ready([f"s{s}" for s in range(S)], False, set())

    with torch.no_grad():
        r = ref_chunks()
        o = ours_chunks()
        t_ref = _time(ref_chunks, flush=flush)
        t_ours = _time(ours_chunks, flush=flush)
    a = torch.cat([x.float() for x in r])
    b = torch.cat([o[f"s{s}"].float().reshape(-1) for s in range(S)])
    n = min(a.numel(), b.numel())
    err = float((a[:n] - b[:n]).norm() / a[:n].norm().clamp_min(1e-12))
    t_state = _stateful_chunk(ours, codes, S, new, flush)
    return {"component": f"Code2Wav streaming chunk, {S} streams x (25 context + 10 new frames)",
            "reference_ms": round(t_ref, 3), "ours_ms": round(t_ours, 3), "speedup": round(t_ref / t_ours, 2),
            "rel_diff": round(err, 4), "ours_stateful_ms": round(t_state, 3),
            "stateful_speedup": round(t_ref / t_state, 2),
            "stateful_note": "kept per-stream state: the 10 new frames only (exact full-sequence output, "
                             "so no rel_diff against the 25-frame-context decode)"}


def _stateful_chunk(ours, codes, S: int, new: int, flush) -> float:
    """One steady 10-frame chunk of every stream through the stateful decoder (graphs
    captured as the vocoder stage does), after three chunks of history per stream."""
    from .models.qwen3_omni.code2wav_stateful import StatefulStreamingCode2Wav

    sc = StatefulStreamingCode2Wav(ours, chunk=new, first_chunk=new, max_streams=S, max_frames=4096)
    sc.capture_graphs()
    rids = [f"s{s}" for s in range(S)]
    for _ in range(3):
        for s in range(S):
            sc.add_codes(rids[s], codes[s, :, :new].t())
        sc.decode_ready(rids)

    def chunk():
        for s in range(S):
            sc.add_codes(rids[s], codes[s, :, :new].t())
        return sc.decode_ready(rids)

    with torch.no_grad():
        return _time(chunk, flush=flush)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-path", default=os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                                       "baseline", "_ref"))
    ap.add_argument("--images", type=int, default=64)
    ap.add_argument("--streams", type=int, default=32)
    args = ap.parse_args()
    _import_reference(args.ref_path)
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with tempfile.TemporaryDirectory() as ckpt:
        _write_checkpoint(ckpt, dev)
        for fn, n in ((audio, args.streams), (vision, args.images), (code2wav, args.streams)):
            try:
                print(json.dumps(fn(ckpt, dev, flush, n)), flush=True)
            except Exception as exc:   # one component failing does not hide the other
                print(json.dumps({"component": fn.__name__, "error": f"{type(exc).__name__}: {exc}"}), flush=True)


if __name__ == "__main__":
    main()
