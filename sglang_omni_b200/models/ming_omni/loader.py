"""Builds (and caches per process) the Ming-Omni components a stage needs:
HF safetensors (``model.*`` LLM, ``audio.*`` / ``linear_proj_audio.*`` tower)
when a checkpoint is given, else random init with fixed seeds and the
fallback tokenizer.  ``overrides`` = {"llm": {...}, "whisper": {...}} shrink
the architecture for tests.  ``ep`` (a ``parallel.EPMoE``) shards the experts
over an expert-parallel group: at full size the LLM's 256 experts (about
200 GB in bf16) need at least two GPUs."""
from __future__ import annotations

import json
import threading

import torch

from ..common.tokenizer import SpecialsByteTokenizer, load_tokenizer
from ..decoder import DecoderLM
from ..weight_loader import has_checkpoint, load_by_prefix
from .audio_encoder import MingAudioEncoder
from .hf_config import (AUDIO_END, AUDIO_PATCH, AUDIO_START, ROLE_ASSISTANT, ROLE_END, ROLE_HUMAN, ROLE_SYSTEM,
                        WhisperConfig, configs_from_hf, llm_config)

_LOCK = threading.Lock()
_CACHE: dict = {}
SEEDS = {"llm": 3, "audio": 13}
SPECIALS = [ROLE_SYSTEM, ROLE_HUMAN, ROLE_ASSISTANT, ROLE_END, AUDIO_START, AUDIO_END, AUDIO_PATCH,
            "<end_of_audio>", "<|endoftext|>"]


def _key(model_path, name, device, overrides):
    return (model_path, name, str(device), json.dumps(overrides or {}, sort_keys=True, default=str))


def _ready(obj):
    """Components are built once and then used from several threads, each on its own
    CUDA stream: finish their initialisation before anyone can see them."""
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()
    return obj


def _cfgs(model_path, overrides):
    c = configs_from_hf(model_path) if has_checkpoint(model_path) else {"llm": llm_config(), "whisper": WhisperConfig()}
    for k, v in ((overrides or {}).get("llm") or {}).items():
        setattr(c["llm"], k, v)
    for k, v in ((overrides or {}).get("whisper") or {}).items():
        setattr(c["whisper"], k, v)
    c["whisper"].out_dim = c["llm"].hidden_size
    return c


def get_tokenizer(model_path: str, overrides: dict | None = None):
    k = _key(model_path, "tok", "cpu", overrides)
    with _LOCK:
        if k not in _CACHE:
            if has_checkpoint(model_path):
                _CACHE[k] = load_tokenizer(model_path)
            else:
                vocab = _cfgs(model_path, overrides)["llm"].vocab_size
                _CACHE[k] = SpecialsByteTokenizer(SPECIALS, vocab, eos="<|endoftext|>")
        return _CACHE[k]


def get_llm(model_path: str, device, overrides: dict | None = None, ep=None) -> DecoderLM:
    k = _key(model_path, "llm", device, overrides) + (id(ep),)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
    cfg = _cfgs(model_path, overrides)["llm"]
    m = DecoderLM(cfg, device, ep=ep)
    if has_checkpoint(model_path):
        load_bailing(m, load_by_prefix(model_path, "model."))
    else:
        m.random_init_(seed=SEEDS["llm"])
    _ready(m)
    with _LOCK:
        _CACHE.setdefault(k, m)
        return _CACHE[k]


def get_audio_encoder(model_path: str, device, overrides: dict | None = None) -> MingAudioEncoder:
    k = _key(model_path, "audio", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
    enc = MingAudioEncoder(_cfgs(model_path, overrides)["whisper"], device)
    if has_checkpoint(model_path):
        sd = load_by_prefix(model_path, "audio.")
        sd = {"audio." + kk: v for kk, v in sd.items()}
        sd.update({"linear_proj_audio." + kk: v for kk, v in load_by_prefix(model_path, "linear_proj_audio.").items()})
        enc.load_hf_state_dict(sd)
    else:
        enc.random_init_(seed=SEEDS["audio"])
    _ready(enc)
    with _LOCK:
        _CACHE.setdefault(k, enc)
        return _CACHE[k]


@torch.no_grad()
def load_bailing(m: DecoderLM, sd: dict[str, torch.Tensor]) -> None:
    """BailingMoeV2 checkpoint names (``model.`` stripped): ``model.word_embeddings``,
    ``layers.N.attention.query_key_value`` / ``dense`` / ``q_norm`` / ``k_norm``,
    ``mlp.gate`` (+ ``expert_bias``), ``mlp.experts.E.*_proj``, ``mlp.shared_experts.*``,
    dense layers' ``mlp.*_proj``, ``lm_head`` (names as remapped in
    sglang_omni/models/ming_omni/thinker.py:558-640)."""
    cfg = m.cfg
    p0 = "model." if any(k.startswith("model.layers.") for k in sd) else ""
    g = lambda k: sd[p0 + k]  # noqa: E731
    cp = lambda dst, src: dst.copy_(src.to(dst.dtype).reshape(dst.shape))  # noqa: E731
    cp(m.embed, g("word_embeddings.weight"))
    e0, El = m.expert0, m.num_local_experts
    for i, L in enumerate(m.layers):
        p = f"layers.{i}."
        cp(L.ln1, g(p + "input_layernorm.weight"))
        cp(L.ln2, g(p + "post_attention_layernorm.weight"))
        cp(L.qkv, g(p + "attention.query_key_value.weight"))
        cp(L.o, g(p + "attention.dense.weight"))
        if cfg.qk_norm:
            for dst, names in ((L.q_norm, ("attention.q_norm.weight", "attention.query_layernorm.weight")),
                               (L.k_norm, ("attention.k_norm.weight", "attention.key_layernorm.weight"))):
                cp(dst, next(sd[p0 + p + n] for n in names if p0 + p + n in sd))
        if cfg.is_moe_layer(i):
            cp(L.router, g(p + "mlp.gate.weight"))
            if hasattr(L, "router_bias"):
                cp(L.router_bias, g(p + "mlp.gate.expert_bias"))
            for j in range(El):
                q = p + f"mlp.experts.{e0 + j}."
                L.w13[j].copy_(torch.cat([g(q + "gate_proj.weight"), g(q + "up_proj.weight")], 0).to(L.w13.dtype))
                L.w2[j].copy_(g(q + "down_proj.weight").to(L.w2.dtype))
            s = p + "mlp.shared_experts."
            cp(L.s13, torch.cat([g(s + "gate_proj.weight"), g(s + "up_proj.weight")], 0))
            cp(L.s2, g(s + "down_proj.weight"))
        else:
            cp(L.mlp13, torch.cat([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")], 0))
            cp(L.mlp2, g(p + "mlp.down_proj.weight"))
    cp(m.final_norm, g("norm.weight"))
    if m.lm_head is not None:
        cp(m.lm_head, sd["lm_head.weight"] if "lm_head.weight" in sd else g("lm_head.weight"))


def eos_ids(model_path: str, overrides: dict | None = None) -> tuple:
    tok = get_tokenizer(model_path, overrides)
    e = getattr(tok, "eos_token_id", None)
    return (int(e),) if e is not None else ()



# ----------------------------------------------------------------------------- talker + AudioVAE
TALKER_SPECIALS = ["<|im_start|>", "<|im_end|>", "<|vision_start|>", "<|vision_pad|>", "<|vision_end|>", "<audio>",
                   "<audioPatch>", "<|endoftext|>"]


def _talker_cfgs(model_path: str, overrides: dict | None):
    """(MingTalkerConfig, AudioVAEConfig) from ``<model>/talker`` (config.json, llm/config.json)
    and ``<model>/talker/vae`` when present, else the defaults; ``overrides`` =
    {"talker": {...}, "talker_llm": {...}, "vae": {...}} shrink them for tests."""
    import os

    from .audio_vae import AudioVAEConfig
    from .talker import MingTalkerConfig

    tdir = os.path.join(model_path, "talker") if model_path else ""
    tc, vc = MingTalkerConfig(), AudioVAEConfig()
    if tdir and os.path.isfile(os.path.join(tdir, "config.json")):
        with open(os.path.join(tdir, "config.json")) as f:
            raw = json.load(f)
        llm = {}
        if os.path.isfile(os.path.join(tdir, "llm", "config.json")):
            with open(os.path.join(tdir, "llm", "config.json")) as f:
                llm = json.load(f)
        tc = MingTalkerConfig.from_dict(raw, llm)
        if os.path.isfile(os.path.join(tdir, "vae", "config.json")):
            with open(os.path.join(tdir, "vae", "config.json")) as f:
                vc = AudioVAEConfig.from_dict(json.load(f))
    ov = overrides or {}
    for k, v in (ov.get("talker") or {}).items():
        setattr(tc, k, v)
    for k, v in (ov.get("talker_llm") or {}).items():
        setattr(tc.llm, k, v)
    for k, v in (ov.get("vae") or {}).items():
        setattr(vc, k, v)
    vc.latent_dim = tc.latent_dim
    return tc, vc, tdir


def get_talker(model_path: str, device, overrides: dict | None = None):
    from .talker import MingTalker

    k = _key(model_path, "talker", device, overrides)
    with _LOCK:
        if k not in _CACHE:
            tc, _, tdir = _talker_cfgs(model_path, overrides)
            m = MingTalker(tc, device=device)
            if tdir and has_checkpoint(tdir):
                m.load_state_dict_ref(load_by_prefix(tdir, ""))
            else:
                m.random_init_(seed=SEEDS["llm"] + 40)
            _CACHE[k] = _ready(m)
        return _CACHE[k]


def get_audio_vae(model_path: str, device, overrides: dict | None = None):
    import os

    from .audio_vae import AudioVAEDecoder

    k = _key(model_path, "vae", device, overrides)
    with _LOCK:
        if k not in _CACHE:
            _, vc, tdir = _talker_cfgs(model_path, overrides)
            m = AudioVAEDecoder(vc, device=device)
            vdir = os.path.join(tdir, "vae") if tdir else ""
            if vdir and has_checkpoint(vdir):
                m.load_state_dict_ref(load_by_prefix(vdir, ""))
            else:
                m.random_init_(seed=SEEDS["llm"] + 41)
            _CACHE[k] = _ready(m)
        return _CACHE[k]


def get_talker_tokenizer(model_path: str, overrides: dict | None = None):
    import os

    k = _key(model_path, "talker_tok", "cpu", overrides)
    with _LOCK:
        if k not in _CACHE:
            tdir = os.path.join(model_path, "talker", "llm") if model_path else ""
            if tdir and os.path.isdir(tdir) and has_checkpoint(os.path.dirname(tdir)):
                _CACHE[k] = load_tokenizer(tdir)
            else:
                tc, _, _ = _talker_cfgs(model_path, overrides)
                _CACHE[k] = SpecialsByteTokenizer(TALKER_SPECIALS, tc.llm.vocab_size, eos="<|endoftext|>")
        return _CACHE[k]
