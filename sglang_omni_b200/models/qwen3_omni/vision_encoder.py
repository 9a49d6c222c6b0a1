"""Qwen3-Omni vision tower on the sm_100a ops.

pixels -> 16x16 (x2 temporal) patches -> patch embedding (the Conv3d as one
tcgen05 GEMM with bias) -> + bilinearly interpolated learned 48x48 position
grid -> 27 x [LN, QKV (bias), 2-D rotary, varlen attention per image, proj,
LN, GELU-tanh MLP] -> 2x2 patch merger (LN, MLP) -> thinker hidden, plus
"deepstack" mergers at layers 8 / 16 / 24 whose outputs are added to the
thinker's hidden states after its first layers.

head_dim 72 runs as 80 in the attention kernel: the per-head q/k/v rows are
padded with zeros at load (scores unchanged, the padded output columns are
zero), and the softmax scale stays 1/sqrt(72).

Architecture: transformers Qwen3OmniMoeVisionEncoder (used by
sglang_omni/models/qwen3_omni/components/image_encoder.py:28-182, which also
swaps the Conv3d patch embedding for an equivalent Linear).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
from torch import nn

from ...preprocessing.vision_grid import (IMAGE_MAX_PIXELS, IMAGE_MIN_PIXELS, VIDEO_MAX_PIXELS, VIDEO_MIN_PIXELS,
                                          resize_grid)
from ... import ops

IMAGE_MEAN = (0.5, 0.5, 0.5)
IMAGE_STD = (0.5, 0.5, 0.5)


@dataclass
class VisionConfig:
    depth: int = 27
    hidden_size: int = 1152
    intermediate_size: int = 4304
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 16
    spatial_merge_size: int = 2
    temporal_patch_size: int = 2
    out_hidden_size: int = 2048
    num_position_embeddings: int = 2304
    deepstack_visual_indexes: list = field(default_factory=lambda: [8, 16, 24])
    dtype: torch.dtype = torch.bfloat16
    # target-size bounds of the checkpoint's image / video processors (preprocessing.vision_grid)
    min_pixels: int = IMAGE_MIN_PIXELS
    max_pixels: int = IMAGE_MAX_PIXELS
    video_min_pixels: int = VIDEO_MIN_PIXELS
    video_max_pixels: int = VIDEO_MAX_PIXELS

    @property
    def head_dim(self):
        return self.hidden_size // self.num_heads

    @property
    def kernel_head_dim(self):
        return ((self.head_dim + 15) // 16) * 16  # 72 -> 80

    @property
    def patch_dim(self):
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2


def _rot_half(x):
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], -1)


class Qwen3OmniVisionEncoder(nn.Module):
    def __init__(self, cfg: VisionConfig | None = None, device="cpu"):
        super().__init__()
        cfg = cfg or VisionConfig()
        self.cfg = cfg
        d, I, dt = cfg.hidden_size, cfg.intermediate_size, cfg.dtype
        nh, hd, kd = cfg.num_heads, cfg.head_dim, cfg.kernel_head_dim
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dt, device=device), requires_grad=False)  # noqa: E731
        self.patch_w, self.patch_b = P(d, cfg.patch_dim), P(d)
        self.pos_embed = P(cfg.num_position_embeddings, d)
        self.blocks = nn.ModuleList()
        for _ in range(cfg.depth):
            B = nn.Module()
            B.n1_w, B.n1_b = P(d), P(d)
            B.qkv_w, B.qkv_b = P(3 * nh * kd, d), P(3 * nh * kd)   # per-head padded to kd
            B.proj_w, B.proj_b = P(d, nh * kd), P(d)
            B.n2_w, B.n2_b = P(d), P(d)
            B.fc1_w, B.fc1_b = P(I, d), P(I)
            B.fc2_w, B.fc2_b = P(d, I), P(d)
            self.blocks.append(B)
        m = cfg.spatial_merge_size ** 2 * d

        def merger(post):
            M = nn.Module()
            M.ln_w, M.ln_b = P(m if post else d), P(m if post else d)
            M.fc1_w, M.fc1_b = P(m, m), P(m)
            M.fc2_w, M.fc2_b = P(cfg.out_hidden_size, m), P(cfg.out_hidden_size)
            return M

        self.merger = merger(False)
        self.deepstack = nn.ModuleList([merger(True) for _ in cfg.deepstack_visual_indexes])
        inv = 1.0 / (10000.0 ** (torch.arange(0, hd // 2, 2, dtype=torch.float32) / (hd // 2)))
        self.register_buffer("inv_freq", inv.to(device), persistent=False)

    @torch.no_grad()
    def random_init_(self, seed: int = 0, std: float = 0.02):
        dev = self.patch_w.device
        for idx, (n, p) in enumerate(self.named_parameters()):
            if n.endswith("_b"):
                p.zero_()
            elif n.split(".")[-1] in ("n1_w", "n2_w", "ln_w"):
                p.fill_(1.0)
            else:
                g = torch.Generator(device=dev).manual_seed(seed * 7331 + idx)
                p.normal_(0.0, std, generator=g)
        self._zero_padding()
        return self

    @torch.no_grad()
    def _zero_padding(self):
        cfg = self.cfg
        nh, hd, kd = cfg.num_heads, cfg.head_dim, cfg.kernel_head_dim
        for B in self.blocks:
            B.qkv_w.view(3, nh, kd, -1)[:, :, hd:] = 0
            B.qkv_b.view(3, nh, kd)[:, :, hd:] = 0
            B.proj_w.view(-1, nh, kd)[:, :, hd:] = 0

    @torch.no_grad()
    def load_hf_state_dict(self, sd: dict[str, torch.Tensor]):
        """``thinker.visual.*`` tensors with the prefix stripped."""
        cfg = self.cfg
        nh, hd, kd, d = cfg.num_heads, cfg.head_dim, cfg.kernel_head_dim, cfg.hidden_size
        c = lambda dst, src: dst.copy_(src.to(dst.dtype))  # noqa: E731
        c(self.patch_w, sd["patch_embed.proj.weight"].reshape(d, -1))
        c(self.patch_b, sd["patch_embed.proj.bias"])
        c(self.pos_embed, sd["pos_embed.weight"])
        for i, B in enumerate(self.blocks):
            p = f"blocks.{i}."
            c(B.n1_w, sd[p + "norm1.weight"]); c(B.n1_b, sd[p + "norm1.bias"])  # noqa: E702
            c(B.n2_w, sd[p + "norm2.weight"]); c(B.n2_b, sd[p + "norm2.bias"])  # noqa: E702
            w = sd[p + "attn.qkv.weight"].view(3, nh, hd, d)
            b = sd[p + "attn.qkv.bias"].view(3, nh, hd)
            B.qkv_w.zero_(); B.qkv_b.zero_()  # noqa: E702
            B.qkv_w.view(3, nh, kd, d)[:, :, :hd] = w.to(B.qkv_w.dtype)
            B.qkv_b.view(3, nh, kd)[:, :, :hd] = b.to(B.qkv_b.dtype)
            B.proj_w.zero_()
            B.proj_w.view(d, nh, kd)[:, :, :hd] = sd[p + "attn.proj.weight"].view(d, nh, hd).to(B.proj_w.dtype)
            c(B.proj_b, sd[p + "attn.proj.bias"])
            c(B.fc1_w, sd[p + "mlp.linear_fc1.weight"]); c(B.fc1_b, sd[p + "mlp.linear_fc1.bias"])  # noqa: E702
            c(B.fc2_w, sd[p + "mlp.linear_fc2.weight"]); c(B.fc2_b, sd[p + "mlp.linear_fc2.bias"])  # noqa: E702
        for M, pre in [(self.merger, "merger.")] + [(m, f"merger_list.{i}.") for i, m in enumerate(self.deepstack)]:
            c(M.ln_w, sd[pre + "ln_q.weight"]); c(M.ln_b, sd[pre + "ln_q.bias"])  # noqa: E702
            c(M.fc1_w, sd[pre + "mlp.0.weight"]); c(M.fc1_b, sd[pre + "mlp.0.bias"])  # noqa: E702
            c(M.fc2_w, sd[pre + "mlp.2.weight"]); c(M.fc2_b, sd[pre + "mlp.2.bias"])  # noqa: E702

    # ------------------------------------------------------------------ positions
    def _per_grid(self, grids, what: str, device) -> torch.Tensor:
        """Interpolated position embeddings ("pos", fp32) or rotary angles ("cos" / "sin", fp32)
        of a batch of grids; each distinct (t, h, w) is computed once and kept (a batch of
        same-size images repeats one grid)."""
        cache = self.__dict__.setdefault("_grid_cache", {})
        parts = []
        for g in grids:
            key = (tuple(int(v) for v in g), str(device))
            hit = cache.get(key)
            if hit is None:
                pe = self._pos_embed([g]).to(device).float()
                c, s_ = self._rope_cos_sin([g], device)
                hit = {"pos": pe, "cos": c.float().contiguous(), "sin": s_.float().contiguous()}
                if len(cache) < 256:
                    cache[key] = hit
            parts.append(hit[what])
        return parts[0] if len(parts) == 1 else torch.cat(parts, 0)

    def _pos_embed(self, grids):
        cfg = self.cfg
        side = int(math.isqrt(cfg.num_position_embeddings))
        ms = cfg.spatial_merge_size
        outs = []
        for t, h, w in grids:
            dev = self.pos_embed.device
            hi = torch.linspace(0, side - 1, h, device=dev)
            wi = torch.linspace(0, side - 1, w, device=dev)
            h0, w0 = hi.long(), wi.long()
            h1, w1 = (h0 + 1).clamp(max=side - 1), (w0 + 1).clamp(max=side - 1)
            dh, dw = hi - h0, wi - w0
            pe = self.pos_embed.float()
            emb = ((1 - dh)[:, None, None] * (1 - dw)[None, :, None] * pe[(h0[:, None] * side + w0[None, :])]
                   + (1 - dh)[:, None, None] * dw[None, :, None] * pe[(h0[:, None] * side + w1[None, :])]
                   + dh[:, None, None] * (1 - dw)[None, :, None] * pe[(h1[:, None] * side + w0[None, :])]
                   + dh[:, None, None] * dw[None, :, None] * pe[(h1[:, None] * side + w1[None, :])])
            emb = emb.repeat(t, 1, 1, 1).view(t, h // ms, ms, w // ms, ms, -1).permute(0, 1, 3, 2, 4, 5)
            outs.append(emb.reshape(-1, emb.shape[-1]))
        return torch.cat(outs, 0)

    def _rope_cos_sin(self, grids, device):
        ms = self.cfg.spatial_merge_size
        coords = []
        for t, h, w in grids:
            r = (torch.arange(h // ms)[:, None, None, None] * ms + torch.arange(ms)[None, None, :, None])
            cl = (torch.arange(w // ms)[None, :, None, None] * ms + torch.arange(ms)[None, None, None, :])
            r = r.expand(h // ms, w // ms, ms, ms).reshape(-1)
            cl = cl.expand(h // ms, w // ms, ms, ms).reshape(-1)
            coords.append(torch.stack([r, cl], -1).repeat(t, 1))
        pos = torch.cat(coords, 0).to(device).float()
        f = torch.cat([pos[:, :1] * self.inv_freq[None], pos[:, 1:] * self.inv_freq[None]], -1)  # [T, hd/2]
        emb = torch.cat([f, f], -1)
        return emb.cos(), emb.sin()

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, patches: torch.Tensor, grids: list[tuple[int, int, int]]):
        """patches [N, patch_dim] (HF patch order), grids [(t, h, w)] -> (embeds [N/4, out], [deepstack ...])."""
        cfg = self.cfg
        dev = self.patch_w.device
        nh, hd, kd, d = cfg.num_heads, cfg.head_dim, cfg.kernel_head_dim, cfg.hidden_size
        x = ops.linear(patches.to(dev, cfg.dtype).contiguous(), self.patch_w, bias=self.patch_b)
        x = (x.float() + self._per_grid(grids, "pos", dev)).to(cfg.dtype)
        cos = self._per_grid(grids, "cos", dev)
        sin = self._per_grid(grids, "sin", dev)
        lens = [t * h * w for t, h, w in grids]
        cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=dev)
        seq_lens = [h * w for t, h, w in grids for _ in range(t)]
        cu_att = torch.tensor([0] + list(np.cumsum(seq_lens)), dtype=torch.int32, device=dev)
        T = x.shape[0]
        ds_out = []
        for li, B in enumerate(self.blocks):
            n1 = ops.layer_norm(x, B.n1_w, B.n1_b, 1e-6)
            qkv = ops.linear(n1, B.qkv_w, bias=B.qkv_b)
            if qkv.is_cuda:
                # RoPE in place on the q and k heads (their padding columns stay zero); q / k / v
                # go to the attention as strided views of the fused rows
                ops.rope_half_inplace(qkv, 2 * nh, kd, hd, cos, sin)
                q, k, v = qkv[:, :nh * kd], qkv[:, nh * kd:2 * nh * kd], qkv[:, 2 * nh * kd:]
            else:
                qkv = qkv.view(T, 3, nh, kd)
                qk = qkv[:, :2, :, :hd].float()
                qk = (qk * cos[:, None, None] + _rot_half(qk) * sin[:, None, None]).to(cfg.dtype)
                q = torch.zeros(T, nh, kd, dtype=cfg.dtype, device=dev)
                k = torch.zeros_like(q)
                q[..., :hd], k[..., :hd] = qk[:, 0], qk[:, 1]
                q, k, v = q.view(T, -1), k.view(T, -1), qkv[:, 2].contiguous().view(T, -1)
            a = ops.varlen_attention(q, k, v, cu_att, nh, nh, kd, scale=1.0 / math.sqrt(hd), q_lens=seq_lens)
            x = ops.linear(a, B.proj_w, bias=B.proj_b, residual=x)
            n2 = ops.layer_norm(x, B.n2_w, B.n2_b, 1e-6)
            f = ops.linear(n2, B.fc1_w, bias=B.fc1_b, act="gelu_tanh")
            x = ops.linear(f, B.fc2_w, bias=B.fc2_b, residual=x)
            if li in cfg.deepstack_visual_indexes:
                M = self.deepstack[cfg.deepstack_visual_indexes.index(li)]
                ds_out.append(self._merge(x, M, post=True))
        return self._merge(x, self.merger, post=False), ds_out

    def _merge(self, x, M, post: bool):
        m = self.cfg.spatial_merge_size ** 2 * self.cfg.hidden_size
        if post:
            h = ops.layer_norm(x.reshape(-1, m).contiguous(), M.ln_w, M.ln_b, 1e-6)
        else:
            h = ops.layer_norm(x, M.ln_w, M.ln_b, 1e-6).reshape(-1, m).contiguous()
        h = ops.linear(h, M.fc1_w, bias=M.fc1_b, act="gelu")
        return ops.linear(h, M.fc2_w, bias=M.fc2_b)


# ----------------------------------------------------------------------------- image processing
def image_to_patches(img: np.ndarray, cfg: VisionConfig, size: int | None = None):
    """uint8 RGB [H, W, 3] -> (patches [N, patch_dim] float32, grid (t, h, w)).

    The image is resized (nearest) to the processor's target size (a multiple of patch*merge
    within the config's pixel bounds, ``vision_grid.resize_grid``), normalised, repeated to the
    temporal patch size, and cut into patches in the merge-block order the encoder expects."""
    p, ms, tp = cfg.patch_size, cfg.spatial_merge_size, cfg.temporal_patch_size
    H, W = img.shape[:2]
    unit = p * ms
    th, tw = (size, size) if size else resize_grid(H, W, unit, cfg.min_pixels, cfg.max_pixels)
    if (th, tw) != (H, W):
        yi = (np.arange(th) * H / th).astype(int)
        xi = (np.arange(tw) * W / tw).astype(int)
        img = img[yi][:, xi]
    x = (img.astype(np.float32) / 255.0 - np.array(IMAGE_MEAN, np.float32)) / np.array(IMAGE_STD, np.float32)
    x = np.repeat(x.transpose(2, 0, 1)[None], tp, 0)  # [tp, C, H, W]
    gh, gw = th // p, tw // p
    x = x.reshape(1, tp, 3, gh // ms, ms, p, gw // ms, ms, p)
    x = x.transpose(0, 3, 6, 4, 7, 2, 1, 5, 8)  # t, bh, bw, mh, mw, C, tp, ph, pw
    return torch.from_numpy(np.ascontiguousarray(x).reshape(gh * gw, -1)), (1, gh, gw)


def images_to_patches_device(images: list[np.ndarray], cfg: VisionConfig, device) -> tuple[torch.Tensor, list]:
    """``image_to_patches`` for a batch on the GPU: the uint8 pixels travel (one pinned copy per
    image shape), the nearest resize, normalisation, temporal repeat and merge-block patch order
    run as device ops.  Returns (patches [sum N_i, patch_dim] fp32 in input order, grids)."""
    p, ms, tp = cfg.patch_size, cfg.spatial_merge_size, cfg.temporal_patch_size
    unit = p * ms
    mean = torch.tensor(IMAGE_MEAN, dtype=torch.float32, device=device)
    std = torch.tensor(IMAGE_STD, dtype=torch.float32, device=device)
    by_shape: dict[tuple, list[int]] = {}
    for i, im in enumerate(images):
        by_shape.setdefault(tuple(im.shape), []).append(i)
    parts: list = [None] * len(images)
    grids: list = [None] * len(images)
    for shape, idxs in by_shape.items():
        H, W = shape[:2]
        th, tw = resize_grid(H, W, unit, cfg.min_pixels, cfg.max_pixels)
        host = torch.from_numpy(np.ascontiguousarray(np.stack([images[i] for i in idxs]))).pin_memory()
        x = host.to(device, non_blocking=True)                                # [b, H, W, 3] uint8
        if (th, tw) != (H, W):
            yi = torch.from_numpy((np.arange(th) * H / th).astype(np.int64)).to(device)
            xi = torch.from_numpy((np.arange(tw) * W / tw).astype(np.int64)).to(device)
            x = x.index_select(1, yi).index_select(2, xi)
        x = (x.float() / 255.0 - mean) / std                                   # [b, th, tw, 3]
        b = x.shape[0]
        gh, gw = th // p, tw // p
        x = x.permute(0, 3, 1, 2)[:, None].expand(b, tp, 3, th, tw)           # [b, tp, C, H, W]
        x = x.reshape(b, tp, 3, gh // ms, ms, p, gw // ms, ms, p)
        x = x.permute(0, 3, 6, 4, 7, 2, 1, 5, 8).reshape(b, gh * gw, -1)      # bh, bw, mh, mw, C, tp, ph, pw
        for j, i in enumerate(idxs):
            parts[i] = x[j]
            grids[i] = (1, gh, gw)
    return torch.cat(parts, 0), grids


def video_to_patches(frames: np.ndarray, cfg: VisionConfig, max_pixels: int | None = None,
                     min_pixels: int | None = None):
    """uint8 RGB frames [N, H, W, 3] (N a multiple of the temporal patch) -> (patches
    [t * gh * gw, patch_dim] float32, grid (t, gh, gw)): every frame resized (nearest) to the
    grid of ``media.video_grid`` (the config's video pixel bounds unless given), normalised,
    consecutive frame pairs forming one temporal patch, cut in the merge-block order of the
    encoder (the image path with t > 1)."""
    from ...preprocessing.media import video_grid

    p, ms, tp = cfg.patch_size, cfg.spatial_merge_size, cfg.temporal_patch_size
    n, H, W = frames.shape[:3]
    t, mh, mw = video_grid(frames, p * ms, cfg.video_max_pixels if max_pixels is None else max_pixels,
                           cfg.video_min_pixels if min_pixels is None else min_pixels)
    th, tw = mh * p * ms, mw * p * ms
    if (th, tw) != (H, W):
        yi = (np.arange(th) * H / th).astype(int)
        xi = (np.arange(tw) * W / tw).astype(int)
        frames = frames[:, yi][:, :, xi]
    x = (frames.astype(np.float32) / 255.0 - np.array(IMAGE_MEAN, np.float32)) / np.array(IMAGE_STD, np.float32)
    x = x[: t * tp].transpose(0, 3, 1, 2)  # [t * tp, C, H, W]
    gh, gw = th // p, tw // p
    x = x.reshape(t, tp, 3, gh // ms, ms, p, gw // ms, ms, p)
    x = x.transpose(0, 3, 6, 4, 7, 2, 1, 5, 8)  # t, bh, bw, mh, mw, C, tp, ph, pw
    return torch.from_numpy(np.ascontiguousarray(x).reshape(t * gh * gw, -1)), (t, gh, gw)


def encode_images(model_path: str, device, images: list, overrides: dict | None = None) -> dict:
    """One vision-tower forward over images (uint8 [H, W, 3]) and videos (``{"frames": uint8
    [N, H, W, 3], ...}`` from ``media.load_video``), in order; per item embeds, deep-stack
    rows and merged (t, h, w) grids."""
    from . import loader

    enc = loader.get_vision_encoder(model_path, device, overrides)
    dev = torch.device(device)
    still = [i for i, im in enumerate(images) if not isinstance(im, dict)]
    patches, grids = [None] * len(images), [None] * len(images)
    if still and dev.type == "cuda":
        # images: patch extraction on the GPU (the host only ships uint8 pixels)
        pt, gs = images_to_patches_device([np.asarray(images[i], dtype=np.uint8) for i in still], enc.cfg, dev)
        ofs = 0
        for i, g in zip(still, gs):
            n = g[0] * g[1] * g[2]
            patches[i], grids[i] = pt[ofs:ofs + n], g
            ofs += n
    for i, im in enumerate(images):
        if patches[i] is not None:
            continue
        if isinstance(im, dict):
            pt, g = video_to_patches(np.asarray(im["frames"], dtype=np.uint8), enc.cfg)
        else:
            pt, g = image_to_patches(np.asarray(im, dtype=np.uint8), enc.cfg)
        patches[i], grids[i] = pt.to(dev), g
    emb, ds = enc(torch.cat(patches, 0), grids)
    ms2 = enc.cfg.spatial_merge_size ** 2
    counts = [t * h * w // ms2 for t, h, w in grids]
    return {"image_embeds": list(torch.split(emb, counts)),
            "deepstack": [list(torch.split(e, counts)) for e in ds],
            "image_grids": [(t, h // enc.cfg.spatial_merge_size, w // enc.cfg.spatial_merge_size)
                            for t, h, w in grids]}
