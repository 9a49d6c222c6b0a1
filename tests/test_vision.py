"""Vision tower against transformers' Qwen3OmniMoeVisionEncoder on CPU."""
import numpy as np
import pytest
import torch

from sglang_omni_b200.models.qwen3_omni.vision_encoder import Qwen3OmniVisionEncoder, VisionConfig, image_to_patches

hf = pytest.importorskip("transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe")
hfc = pytest.importorskip("transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe")


def tiny():
    cfg = hfc.Qwen3OmniMoeVisionEncoderConfig(depth=3, hidden_size=64, intermediate_size=96, num_heads=4,
                                              patch_size=4, spatial_merge_size=2, temporal_patch_size=2,
                                              out_hidden_size=40, num_position_embeddings=64,
                                              deepstack_visual_indexes=[0, 2])
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    m = hf.Qwen3OmniMoeVisionEncoder(cfg).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(torch.randn_like(p) * (0.1 if p.dim() > 1 else 0.02) + (1.0 if ("norm" in n or "ln" in n)
                                                                             and n.endswith("weight") else 0.0))
    ours = Qwen3OmniVisionEncoder(VisionConfig(depth=3, hidden_size=64, intermediate_size=96, num_heads=4,
                                               patch_size=4, out_hidden_size=40, num_position_embeddings=64,
                                               deepstack_visual_indexes=[0, 2], dtype=torch.float32))
    ours.load_hf_state_dict(m.state_dict())
    return m, ours


def test_vision_matches_hf_cpu():
    m, ours = tiny()
    rng = np.random.default_rng(0)
    imgs = [rng.integers(0, 256, (16, 24, 3), dtype=np.uint8), rng.integers(0, 256, (8, 8, 3), dtype=np.uint8)]
    patches, grids = zip(*[image_to_patches(im, ours.cfg) for im in imgs])
    px = torch.cat(patches, 0)
    grid = torch.tensor(grids)
    with torch.no_grad():
        ref = m(px, grid_thw=grid)
        out, ds = ours(px, list(grids))
    ref_main = ref.pooler_output if getattr(ref, "pooler_output", None) is not None else ref.last_hidden_state
    ref_ds = ref.deepstack_features
    assert out.shape == ref_main.shape
    assert (out - ref_main).abs().max() / ref_main.abs().max() < 1e-3
    for a, b in zip(ds, ref_ds):
        assert (a - b).abs().max() / b.abs().max() < 1e-3


@pytest.mark.gpu
def test_vision_gpu_matches_cpu_head_dim_72():
    """head_dim 72 (the real tower's) runs as 80 in the attention kernel."""
    cfg = dict(depth=2, hidden_size=288, intermediate_size=512, num_heads=4, out_hidden_size=256,
               deepstack_visual_indexes=[0])
    cpu = Qwen3OmniVisionEncoder(VisionConfig(**cfg, dtype=torch.float32)).random_init_(seed=2, std=0.05)
    gpu = Qwen3OmniVisionEncoder(VisionConfig(**cfg), device="cuda")
    with torch.no_grad():
        for (n, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
    rng = np.random.default_rng(1)
    img = rng.integers(0, 256, (128, 96, 3), dtype=np.uint8)
    px, grid = image_to_patches(img, cpu.cfg)
    ref, ref_ds = cpu(px, [grid])
    out, ds = gpu(px, [grid])
    assert (out.float().cpu() - ref).abs().max() / ref.abs().max() < 0.05
    assert (ds[0].float().cpu() - ref_ds[0]).abs().max() / ref_ds[0].abs().max() < 0.05


def test_vision_video_matches_hf_cpu():
    """A 4-frame clip (two temporal patches) through our patching + tower and HF's."""
    from sglang_omni_b200.models.qwen3_omni.vision_encoder import video_to_patches

    m, ours = tiny()
    rng = np.random.default_rng(3)
    frames = rng.integers(0, 256, (4, 16, 24, 3), dtype=np.uint8)
    px, grid = video_to_patches(frames, ours.cfg, max_pixels=16 * 24, min_pixels=16)
    assert grid == (2, 4, 6)
    with torch.no_grad():
        ref = m(px, grid_thw=torch.tensor([grid]))
        out, ds = ours(px, [grid])
    ref_main = ref.pooler_output if getattr(ref, "pooler_output", None) is not None else ref.last_hidden_state
    assert (out - ref_main).abs().max() / ref_main.abs().max() < 1e-3


@pytest.mark.gpu
def test_device_patch_extraction_matches_host():
    """Images patchified on the GPU (batched per shape, nearest resize included) equal the host
    path, in input order."""
    import numpy as np

    from sglang_omni_b200.models.qwen3_omni.vision_encoder import (VisionConfig, image_to_patches,
                                                                    images_to_patches_device)

    cfg = VisionConfig()
    rng = np.random.default_rng(0)
    imgs = [rng.integers(0, 256, s, dtype=np.uint8) for s in [(448, 448, 3), (300, 500, 3), (448, 448, 3), (64, 96, 3)]]
    got, grids = images_to_patches_device(imgs, cfg, torch.device("cuda", 0))
    refs = [image_to_patches(im, cfg) for im in imgs]
    assert grids == [g for _, g in refs]
    ref = torch.cat([p for p, _ in refs], 0)
    torch.testing.assert_close(got.cpu(), ref, atol=1e-6, rtol=1e-6)


def test_resize_grid_matches_the_hf_processor_rule():
    """Target sizes of images / video frames equal transformers' Qwen2-VL-family smart_resize
    (token counts match the processor the checkpoint was trained with), and the checkpoint's
    processor configs set the bounds."""
    import json
    import random

    from transformers.models.qwen2_vl.image_processing_qwen2_vl import smart_resize

    from sglang_omni_b200.preprocessing.vision_grid import checkpoint_bounds, resize_grid

    rnd = random.Random(0)
    for _ in range(3000):
        h, w = rnd.randint(16, 5000), rnd.randint(16, 5000)
        if max(h, w) > 200 * min(h, w):
            continue
        f, lo, hi = rnd.choice([28, 32]), rnd.choice([3136, 131072]), rnd.choice([786432, 12845056])
        assert tuple(smart_resize(h, w, f, lo, hi)) == resize_grid(h, w, f, lo, hi), (h, w, f, lo, hi)
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        with open(f"{d}/preprocessor_config.json", "w") as fh:
            json.dump({"min_pixels": 1000, "max_pixels": 2000000}, fh)
        with open(f"{d}/video_preprocessor_config.json", "w") as fh:
            json.dump({"size": {"shortest_edge": 4096, "longest_edge": 90000}}, fh)
        b = checkpoint_bounds(d)
        assert (b.image_min, b.image_max, b.video_min, b.video_max) == (1000, 2000000, 4096, 90000)
