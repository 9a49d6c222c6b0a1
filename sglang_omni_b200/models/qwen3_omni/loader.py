"""Builds (and caches per process) the Qwen3-Omni components a stage needs.

With a checkpoint directory (HF safetensors) every component loads its own
key prefix; otherwise components are random-initialised with fixed per-
component seeds, so two processes (e.g. thinker and talker stages on
different GPUs) regenerate identical tensors (the talker needs the thinker's
token-embedding rows, as the reference reads them from safetensors in
sglang_omni/models/qwen3_omni/components/talker_executor.py:68-97).
``overrides`` shrink architectures for tests (e.g. {"thinker": {"num_layers": 2}}).
"""
from __future__ import annotations

import json
import threading

import torch

from ..decoder import DecoderLM
from ..weight_loader import has_checkpoint, load_by_prefix, load_decoder_from_hf
from .audio_encoder import AudioEncoderConfig, Qwen3OmniAudioEncoder
from .code2wav import Code2Wav, Code2WavConfig
from .hf_config import code_predictor_config, configs_from_hf, talker_text_config, thinker_text_config
from .talker import Qwen3OmniTalker

_LOCK = threading.Lock()
_CACHE: dict[tuple, object] = {}

SEEDS = {"thinker": 0, "talker": 11, "audio": 21, "code2wav": 31, "vision": 41}


def _key(model_path, name, device, overrides):
    return (model_path, name, str(device), json.dumps(overrides or {}, sort_keys=True, default=str))


def _ready(obj):
    """Components are built once and then used from several threads, each on its own
    CUDA stream: finish their initialisation before anyone can see them."""
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()
    return obj


def _cfgs(model_path):
    if has_checkpoint(model_path):
        return configs_from_hf(model_path)
    return {"thinker": thinker_text_config(), "talker": talker_text_config(),
            "code_predictor": code_predictor_config()}


def _apply(cfg, over: dict | None):
    for k, v in (over or {}).items():
        if k == "dtype" and isinstance(v, str):   # YAML configs name dtypes ("float32", "bfloat16")
            v = getattr(torch, v.replace("torch.", ""))
        setattr(cfg, k, v)
    return cfg


def get_thinker(model_path: str, device, overrides: dict | None = None) -> DecoderLM:
    k = _key(model_path, "thinker", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
        cfg = _apply(_cfgs(model_path)["thinker"], (overrides or {}).get("thinker"))
        m = DecoderLM(cfg, device=device)
        if has_checkpoint(model_path):
            sd = load_by_prefix(model_path, "thinker.")
            load_decoder_from_hf(m, sd, "model.", "lm_head.weight")
        else:
            m.random_init_(seed=SEEDS["thinker"])
        _ready(m)
        _CACHE[k] = m
        return m


def build_thinker_rank(args: dict, rank: int, world: int, device, group, mode: str) -> DecoderLM:
    """One rank of a thinker stage group (``parallel.rank_group``): ``tp`` holds this
    rank's heads / expert slice / MLP slices with the fused TP reduce points, ``ep``
    this rank's experts with the fused EP exchange (data-parallel attention; with
    ``args["tp"]`` > 1 the attention is tensor parallel inside groups of that many
    ranks), the other modes a full copy.  Weights: the checkpoint's slices, or the same
    deterministic random init as the single-GPU thinker."""
    model_path = args.get("model_path", "")
    cfg = _apply(_cfgs(model_path)["thinker"], (args.get("overrides") or {}).get("thinker"))
    max_tokens = int(args.get("max_tokens", 8192))
    tp_size = int(args.get("tp", 1))
    tp = ep = None
    if mode == "tp":
        from ...parallel.tp import TPGroup

        tp = TPGroup(cfg.hidden_size, max_tokens, device, group=group)
    elif mode == "ep":
        from ...parallel.ep_moe import EPMoE

        if tp_size > 1:   # attention TP inside this rank's data-parallel group, EP over every rank
            from ...parallel.tp import TPGroup

            g0 = rank // tp_size * tp_size
            sub = group.subgroup(list(range(g0, g0 + tp_size)), f"tp{g0 // tp_size}")
            tp = TPGroup(cfg.hidden_size, max_tokens, device, group=sub)
        ep = EPMoE(cfg.num_experts, cfg.topk, cfg.hidden_size, cfg.moe_intermediate_size, max_tokens=max_tokens,
                   device=device, group=group)
    m = DecoderLM(cfg, device=device, tp=tp, ep=ep)
    if has_checkpoint(model_path):
        load_decoder_from_hf(m, load_by_prefix(model_path, "thinker."), "model.", "lm_head.weight")
    else:
        m.random_init_(seed=SEEDS["thinker"])
    return _ready(m)


def thinker_embedding(model_path: str, device, overrides: dict | None = None) -> torch.Tensor:
    """The thinker's token-embedding table without building the whole thinker
    (reuses the thinker if this process already has it)."""
    k = _key(model_path, "thinker", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k].embed
    cfg = _apply(_cfgs(model_path)["thinker"], (overrides or {}).get("thinker"))
    if has_checkpoint(model_path):
        sd = load_by_prefix(model_path, "thinker.model.embed_tokens.")
        return sd["weight"].to(device, cfg.dtype)
    # parameter 0 of DecoderLM.random_init_ (the embedding) with the thinker seed
    t = torch.empty(cfg.vocab_size, cfg.hidden_size, dtype=cfg.dtype, device=device)
    g = torch.Generator(device=torch.device(device)).manual_seed(SEEDS["thinker"] * 100003 + 0)
    return t.normal_(0.0, 0.02, generator=g)


def get_talker(model_path: str, device, overrides: dict | None = None) -> Qwen3OmniTalker:
    k = _key(model_path, "talker", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
        cfgs = _cfgs(model_path)
        tcfg = _apply(cfgs.get("talker", talker_text_config()), (overrides or {}).get("talker"))
        ccfg = _apply(cfgs.get("code_predictor", code_predictor_config()), (overrides or {}).get("code_predictor"))
        thinker_hidden = _apply(cfgs["thinker"], (overrides or {}).get("thinker")).hidden_size
        t = Qwen3OmniTalker(tcfg, ccfg, thinker_hidden=thinker_hidden, device=device)
        if has_checkpoint(model_path):
            sd = load_by_prefix(model_path, "talker.")
            load_decoder_from_hf(t.lm, sd, "model.", "codec_head.weight", embed_key="codec_embedding.weight")
            with torch.no_grad():
                for dst, key in [(t.text_fc1_w, "text_projection.linear_fc1.weight"),
                                 (t.text_fc1_b, "text_projection.linear_fc1.bias"),
                                 (t.text_fc2_w, "text_projection.linear_fc2.weight"),
                                 (t.text_fc2_b, "text_projection.linear_fc2.bias"),
                                 (t.hid_fc1_w, "hidden_projection.linear_fc1.weight"),
                                 (t.hid_fc1_b, "hidden_projection.linear_fc1.bias"),
                                 (t.hid_fc2_w, "hidden_projection.linear_fc2.weight"),
                                 (t.hid_fc2_b, "hidden_projection.linear_fc2.bias")]:
                    dst.copy_(sd[key].to(dst.dtype))
                cp = {kk[len("code_predictor."):]: v for kk, v in sd.items() if kk.startswith("code_predictor.")}
                load_decoder_from_hf(t.cp, cp, "model.", None, embed_key="__none__")
                for gidx in range(t.cp_heads.shape[0]):
                    t.cp_heads[gidx].copy_(cp[f"lm_head.{gidx}.weight"].to(t.cp_heads.dtype))
                    t.cp_embeds[gidx].copy_(cp[f"model.codec_embedding.{gidx}.weight"].to(t.cp_embeds.dtype))
        else:
            t.random_init_(seed=SEEDS["talker"])
        _ready(t)
        _CACHE[k] = t
        return t


def get_audio_encoder(model_path: str, device, overrides: dict | None = None) -> Qwen3OmniAudioEncoder:
    k = _key(model_path, "audio", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
        cfg = AudioEncoderConfig()
        thinker_hidden = _apply(_cfgs(model_path)["thinker"], (overrides or {}).get("thinker")).hidden_size
        cfg.output_dim = thinker_hidden
        _apply(cfg, (overrides or {}).get("audio"))
        m = Qwen3OmniAudioEncoder(cfg, device)
        if has_checkpoint(model_path):
            m.load_hf_state_dict(load_by_prefix(model_path, "thinker.audio_tower."))
        else:
            m.random_init_(seed=SEEDS["audio"])
        _ready(m)
        _CACHE[k] = m
        return m


def vision_config(model_path: str, overrides: dict | None = None):
    """The vision tower's config: defaults, the checkpoint processors' resize bounds, then the
    ``vision`` overrides (preprocessing builds the same one, so token grids agree)."""
    from ...preprocessing.vision_grid import checkpoint_bounds
    from .vision_encoder import VisionConfig

    b = checkpoint_bounds(model_path)
    cfg = VisionConfig(min_pixels=b.image_min, max_pixels=b.image_max, video_min_pixels=b.video_min,
                       video_max_pixels=b.video_max)
    return _apply(cfg, (overrides or {}).get("vision"))


def get_vision_encoder(model_path: str, device, overrides: dict | None = None):
    from .vision_encoder import Qwen3OmniVisionEncoder

    k = _key(model_path, "vision", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
        cfg = vision_config(model_path, overrides)
        if "out_hidden_size" not in ((overrides or {}).get("vision") or {}):
            cfg.out_hidden_size = _apply(_cfgs(model_path)["thinker"], (overrides or {}).get("thinker")).hidden_size
        m = Qwen3OmniVisionEncoder(cfg, device)
        if has_checkpoint(model_path):
            m.load_hf_state_dict(load_by_prefix(model_path, "thinker.visual."))
        else:
            m.random_init_(seed=SEEDS["vision"])
        _ready(m)
        _CACHE[k] = m
        return m


def get_code2wav(model_path: str, device, overrides: dict | None = None) -> Code2Wav:
    k = _key(model_path, "code2wav", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
        cfg = _apply(Code2WavConfig(), (overrides or {}).get("code2wav"))
        m = Code2Wav(cfg, device)
        if has_checkpoint(model_path):
            m.load_hf_state_dict(load_by_prefix(model_path, "code2wav."))
        else:
            m.random_init_(seed=SEEDS["code2wav"])
        _ready(m)
        _CACHE[k] = m
        return m
