"""Hub repository ids as model paths: cache first, download when online, a partial cached
snapshot fetched again, clear errors offline; local paths and synthetic names untouched
(snapshot_download replaced by a fake: no network here)."""
import json
import os

import pytest

from sglang_omni_b200.models import model_path as mp


@pytest.fixture
def fake_hub(tmp_path, monkeypatch):
    import huggingface_hub

    calls = []
    state = {"cached": None, "remote": None}

    def snapshot_download(repo, local_files_only=False, force_download=False, **_):
        calls.append((repo, local_files_only, force_download))
        if local_files_only:
            if state["cached"] is None:
                raise FileNotFoundError("not cached")
            return state["cached"]
        return state["remote"]

    monkeypatch.setattr(huggingface_hub, "snapshot_download", snapshot_download)
    monkeypatch.delenv("HF_HUB_OFFLINE", raising=False)
    mp._RESOLVED.clear()
    return calls, state, tmp_path


def _ckpt(d, shards=("a.safetensors", "b.safetensors"), present=None):
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump({"architectures": ["Qwen3ForCausalLM"]}, f)
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": {f"w{i}": s for i, s in enumerate(shards)}}, f)
    for s in (shards if present is None else present):
        open(os.path.join(d, s), "wb").close()
    return str(d)


def test_local_and_synthetic_paths_pass_through(fake_hub, tmp_path):
    calls, _, _ = fake_hub
    for p in ("", "random", "toy", str(tmp_path), "relative/dir/that/does/not/exist"):
        assert mp.resolve_model_path(p) == p
    assert calls == []


def test_cached_snapshot_used_without_network(fake_hub):
    calls, state, tmp = fake_hub
    state["cached"] = _ckpt(tmp / "cache")
    assert mp.resolve_model_path("Org/Model-1") == state["cached"]
    assert calls == [("Org/Model-1", True, False)]
    assert mp.resolve_model_path("Org/Model-1") == state["cached"] and len(calls) == 1   # memoised


def test_partial_snapshot_refetched_once(fake_hub):
    calls, state, tmp = fake_hub
    state["cached"] = _ckpt(tmp / "cache", present=["a.safetensors"])        # b.safetensors missing
    state["remote"] = _ckpt(tmp / "fresh")
    assert mp.resolve_model_path("Org/Model-2") == state["remote"]
    assert calls[-1] == ("Org/Model-2", False, True)


def test_download_when_not_cached_and_offline_errors(fake_hub, monkeypatch):
    calls, state, tmp = fake_hub
    state["remote"] = _ckpt(tmp / "dl")
    assert mp.resolve_model_path("Org/Model-3") == state["remote"]
    assert calls[-1] == ("Org/Model-3", False, False)
    monkeypatch.setenv("HF_HUB_OFFLINE", "1")
    with pytest.raises(FileNotFoundError, match="offline"):
        mp.resolve_model_path("Org/Model-4")


def test_config_manager_reads_the_resolved_snapshot(fake_hub):
    from sglang_omni_b200.config import ConfigManager

    _, state, tmp = fake_hub
    state["cached"] = _ckpt(tmp / "c2")
    cfg = ConfigManager.from_model_path("Org/Qwen3-Tiny")
    assert type(cfg).__name__ == "HFTextPipelineConfig" and cfg.model_path == "Org/Qwen3-Tiny"
