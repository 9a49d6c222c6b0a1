"""HF parity of the decoders on CPU: our ``DecoderLM`` (the thinker and the talker
backbone) and the M-RoPE position builder against transformers' Qwen3-Omni
modules at tiny sizes, with the same random weights.

* thinker text model: ``Qwen3OmniMoeThinkerTextModel`` (GQA, QK-norm,
  interleaved M-RoPE with distinct t/h/w positions, softmax top-k MoE);
* talker text model: ``Qwen3OmniMoeTalkerModel`` (MoE + sigmoid-gated shared
  expert);
* M-RoPE positions of an audio + image + text prompt: ``get_rope_index`` of
  ``Qwen3OmniMoeThinkerForConditionalGeneration``.
"""
import math

import pytest
import torch

from sglang_omni_b200.engines.ar import KVPool
from sglang_omni_b200.models.decoder import DecoderConfig, DecoderLM, ForwardBatch
from sglang_omni_b200.models.weight_loader import load_decoder_from_hf
from sglang_omni_b200.ops import prefill_tiles

hm = pytest.importorskip("transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe")
hc = pytest.importorskip("transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe")

V, H, L, NH, NKV, HD, E, K, I = 300, 64, 2, 4, 2, 16, 8, 2, 24
SECTION = [2, 3, 3]


def _randomise(m, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("norm.weight") or "layernorm" in n:
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * (0.5 / math.sqrt(p.shape[-1])))


def _ours_forward(model, tokens, positions):
    """Final normed hidden states of one prefill of `tokens` at M-RoPE `positions` [3, T]."""
    cfg = model.cfg
    T = len(tokens)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, (T + 63) // 64 + 2, "cpu", torch.float32)
    pages = pool.alloc((T + 63) // 64)
    t = torch.arange(T)
    slots = (torch.tensor(pages)[t // 64] * 64 + t % 64).to(torch.int32)
    req, tok0 = prefill_tiles([T], cfg.num_heads // cfg.num_kv_heads)
    fb = ForwardBatch(is_decode=False, positions=positions.to(torch.int32), slot_mapping=slots,
                      kv_lens=torch.tensor([T], dtype=torch.int32), block_table=torch.tensor([pages], dtype=torch.int32),
                      input_ids=torch.tensor(tokens, dtype=torch.int32), cu_q=torch.tensor([0, T], dtype=torch.int32),
                      tile_req=torch.tensor(req, dtype=torch.int32), tile_tok0=torch.tensor(tok0, dtype=torch.int32))
    with torch.no_grad():
        return model(fb, pool.kv).float()


def _positions(T):
    """Distinct t / h / w rows (an image-like block in the middle), so the interleaving matters."""
    p = torch.arange(T).repeat(3, 1)
    p[1, 10:26] = 10 + torch.arange(16) // 4
    p[2, 10:26] = 10 + torch.arange(16) % 4
    p[0, 10:26] = 10
    p[:, 26:] = p[:, 26:] - 16 + 4
    return p


def _rope_params():
    return {"rope_type": "default", "rope_theta": 10000.0, "mrope_section": SECTION, "interleaved": True,
            "mrope_interleaved": True}


def test_thinker_text_model_matches_hf():
    cfg = hc.Qwen3OmniMoeTextConfig(vocab_size=V, hidden_size=H, intermediate_size=96, num_hidden_layers=L,
                                    num_attention_heads=NH, num_key_value_heads=NKV, head_dim=HD, num_experts=E,
                                    num_experts_per_tok=K, moe_intermediate_size=I, rope_scaling=_rope_params(),
                                    rope_theta=10000.0, decoder_sparse_step=1, mlp_only_layers=[],
                                    norm_topk_prob=True, rms_norm_eps=1e-6)
    cfg._attn_implementation = "eager"
    ref = hm.Qwen3OmniMoeThinkerTextModel(cfg).eval()
    _randomise(ref, 0)
    ours = DecoderLM(DecoderConfig(vocab_size=V, hidden_size=H, num_layers=L, num_heads=NH, num_kv_heads=NKV,
                                   head_dim=HD, intermediate_size=96, num_experts=E, topk=K, moe_intermediate_size=I,
                                   norm_topk_prob=True, rms_norm_eps=1e-6, rope_theta=10000.0, mrope_section=SECTION,
                                   mrope_interleaved=True, qk_norm=True, max_position=4096, dtype=torch.float32))
    load_decoder_from_hf(ours, dict(ref.state_dict()), model_prefix="", lm_head_key=None)
    T = 40
    tokens = torch.randint(0, V, (T,), generator=torch.Generator().manual_seed(3)).tolist()
    pos = _positions(T)
    with torch.no_grad():
        r = ref(input_ids=torch.tensor([tokens]), position_ids=pos[:, None, :]).last_hidden_state[0].float()
    o = _ours_forward(ours, tokens, pos)
    assert o.shape == r.shape
    err = float((o - r).norm() / r.norm())
    assert err < 1e-4, err


def test_talker_text_model_matches_hf():
    tc = hc.Qwen3OmniMoeTalkerTextConfig(vocab_size=V, hidden_size=H, intermediate_size=96, num_hidden_layers=L,
                                         num_attention_heads=NH, num_key_value_heads=NKV, head_dim=HD, num_experts=E,
                                         num_experts_per_tok=K, moe_intermediate_size=I,
                                         shared_expert_intermediate_size=40, rope_scaling=_rope_params(),
                                         rope_theta=10000.0, decoder_sparse_step=1, mlp_only_layers=[],
                                         norm_topk_prob=True, rms_norm_eps=1e-6)
    tc._attn_implementation = "eager"
    ref = hm.Qwen3OmniMoeTalkerModel(tc).eval()
    _randomise(ref, 1)
    ours = DecoderLM(DecoderConfig(vocab_size=V, hidden_size=H, num_layers=L, num_heads=NH, num_kv_heads=NKV,
                                   head_dim=HD, intermediate_size=96, num_experts=E, topk=K, moe_intermediate_size=I,
                                   shared_expert_intermediate_size=40, shared_expert_gate=True, norm_topk_prob=True,
                                   rms_norm_eps=1e-6, rope_theta=10000.0, mrope_section=SECTION,
                                   mrope_interleaved=True, qk_norm=True, max_position=4096, dtype=torch.float32))
    sd = {k.replace("codec_embedding.", "embed_tokens."): v for k, v in ref.state_dict().items()}
    load_decoder_from_hf(ours, sd, model_prefix="", lm_head_key=None)
    T = 40
    tokens = torch.randint(0, V, (T,), generator=torch.Generator().manual_seed(4)).tolist()
    pos = _positions(T)
    emb = ours.embed[torch.tensor(tokens)].float()
    with torch.no_grad():
        r = ref(inputs_embeds=emb[None], position_ids=pos[:, None, :]).last_hidden_state[0].float()
    o = _ours_forward(ours, tokens, pos)
    err = float((o - r).norm() / r.norm())
    assert err < 1e-4, err


def test_mrope_positions_match_hf_get_rope_index():
    """Audio + image + text prompt: our layout's [3, L] positions and decode delta equal
    transformers' get_rope_index on the same ids (image grid in patches, audio as mel frames)."""
    import types

    from sglang_omni_b200.models.qwen3_omni import engine_io as eio
    from sglang_omni_b200.models.qwen3_omni.hf_config import (AUDIO_START_TOKEN_ID, AUDIO_TOKEN_ID, IMAGE_TOKEN_ID,
                                                              VIDEO_TOKEN_ID, VISION_START_TOKEN_ID)

    cls = hm.Qwen3OmniMoePreTrainedModelForConditionalGeneration
    fake = types.SimpleNamespace(
        config=types.SimpleNamespace(image_token_id=IMAGE_TOKEN_ID, video_token_id=VIDEO_TOKEN_ID,
                                     audio_token_id=AUDIO_TOKEN_ID, vision_start_token_id=VISION_START_TOKEN_ID,
                                     audio_start_token_id=AUDIO_START_TOKEN_ID, position_id_per_seconds=25),
        spatial_merge_size=2)
    fake.get_llm_pos_ids_for_vision = types.MethodType(cls.get_llm_pos_ids_for_vision, fake)

    class Tok:
        def encode(self, s):
            return [1000 + (ord(c) % 50) for c in s]

    mel = 997  # audio feature frames -> tokens after the 8x downsample
    n_audio = int(hm._get_feat_extract_output_lengths(torch.tensor(mel)))
    for grids in ([(1, 4, 6)], [(1, 4, 6), (1, 3, 5)]):
        lay = eio.build_prompt(Tok(), None, "describe both", [n_audio], image_grids=grids, system="be brief")
        ours, delta = eio.mrope_positions(lay)
        patches = torch.tensor([[t, 2 * h, 2 * w] for (t, h, w) in grids])
        ids = torch.tensor([lay.ids])
        ref, ref_delta = cls.get_rope_index(fake, ids, image_grid_thw=patches, audio_seqlens=torch.tensor([mel]),
                                            attention_mask=torch.ones_like(ids))
        assert torch.equal(ours.long(), ref[:, 0].long()), (ours, ref[:, 0])
        assert delta == int(ref_delta[0])


def test_code_predictor_backbone_matches_hf():
    """The code predictor's dense decoder (1-D RoPE, QK-norm, SiLU MLP) against
    ``Qwen3OmniMoeTalkerCodePredictorModel`` on the same input embeddings."""
    c = hc.Qwen3OmniMoeTalkerCodePredictorConfig(vocab_size=V, hidden_size=H, intermediate_size=96, num_hidden_layers=L,
                                                 num_attention_heads=NH, num_key_value_heads=NKV, head_dim=HD,
                                                 num_code_groups=4, rope_theta=10000.0, rms_norm_eps=1e-6)
    c._attn_implementation = "eager"
    ref = hm.Qwen3OmniMoeTalkerCodePredictorModel(c).eval()
    _randomise(ref, 2)
    ours = DecoderLM(DecoderConfig(vocab_size=V, hidden_size=H, num_layers=L, num_heads=NH, num_kv_heads=NKV,
                                   head_dim=HD, intermediate_size=96, rms_norm_eps=1e-6, rope_theta=10000.0,
                                   qk_norm=True, max_position=64, dtype=torch.float32))
    sd = {k: v for k, v in ref.state_dict().items() if not k.startswith("codec_embedding.")}
    sd["embed_tokens.weight"] = ref.state_dict()["codec_embedding.0.weight"]
    load_decoder_from_hf(ours, sd, model_prefix="", lm_head_key=None)
    T = 17   # a talker hidden state + 16 code groups
    tokens = torch.randint(0, V, (T,), generator=torch.Generator().manual_seed(5)).tolist()
    pos = torch.arange(T).repeat(3, 1)
    emb = ours.embed[torch.tensor(tokens)].float()
    with torch.no_grad():
        r = ref(inputs_embeds=emb[None], position_ids=torch.arange(T)[None]).last_hidden_state[0].float()
    o = _ours_forward(ours, tokens, pos)
    err = float((o - r).norm() / r.norm())
    assert err < 1e-4, err


def test_mrope_video_positions_match_hf_get_rope_index():
    """Image + video + audio prompt (2 fps sampling: 1 s per temporal patch)."""
    import types

    from sglang_omni_b200.models.qwen3_omni import engine_io as eio
    from sglang_omni_b200.models.qwen3_omni.hf_config import (AUDIO_START_TOKEN_ID, AUDIO_TOKEN_ID, IMAGE_TOKEN_ID,
                                                              VIDEO_TOKEN_ID, VISION_START_TOKEN_ID)

    cls = hm.Qwen3OmniMoePreTrainedModelForConditionalGeneration
    fake = types.SimpleNamespace(
        config=types.SimpleNamespace(image_token_id=IMAGE_TOKEN_ID, video_token_id=VIDEO_TOKEN_ID,
                                     audio_token_id=AUDIO_TOKEN_ID, vision_start_token_id=VISION_START_TOKEN_ID,
                                     audio_start_token_id=AUDIO_START_TOKEN_ID, position_id_per_seconds=25),
        spatial_merge_size=2)
    fake.get_llm_pos_ids_for_vision = types.MethodType(cls.get_llm_pos_ids_for_vision, fake)

    class Tok:
        def encode(self, s):
            return [1000 + (ord(c) % 50) for c in s]

    mel = 500
    n_audio = int(hm._get_feat_extract_output_lengths(torch.tensor(mel)))
    for spg in (1.0, 2.0):
        lay = eio.build_prompt(Tok(), None, "what happens", [n_audio], image_grids=[(1, 3, 4)],
                               video_grids=[(3, 2, 3)], video_second_per_grid=[spg])
        ours, delta = eio.mrope_positions(lay)
        ids = torch.tensor([lay.ids])
        ref, ref_delta = cls.get_rope_index(fake, ids, image_grid_thw=torch.tensor([[1, 6, 8]]),
                                            video_grid_thw=torch.tensor([[3, 4, 6]]),
                                            audio_seqlens=torch.tensor([mel]), attention_mask=torch.ones_like(ids),
                                            second_per_grids=torch.tensor([spg]))
        assert torch.equal(ours.long(), ref[:, 0].long()), (spg, ours, ref[:, 0])
        assert delta == int(ref_delta[0])
