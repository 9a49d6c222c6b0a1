"""Pipeline configs written by the reference's ``config export`` command
(sglang_omni/cli/config.py:45-76: ``config_cls(model_path=...).model_dump(mode="json")`` dumped as
YAML) load here unchanged, every dotted name in them resolves, and the speech layout compiles and
serves a request once its devices and model sizes are overridden the way a user would override
them on the command line (``--stages.4.executor.args.device cpu``).

The export runs in a child interpreter against the reference installed under ``baseline/_ref`` (the
test is skipped when it is not installed): the reference package's media decoders import libraries
this image lacks (PyAV, librosa, ...), so placeholder modules stand in for whichever is missing;
building a config object never calls them.  CPU only.
"""
import asyncio
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

EXPORT = textwrap.dedent("""
    import importlib, importlib.machinery, sys
    import yaml
    sys.path.insert(0, sys.argv[1])
    from sglang_omni_b200.bench_components import _Placeholder
    import transformers  # noqa: F401  (its optional-package probes run before any placeholder exists)
    sys.path.insert(0, sys.argv[2])

    def load(name):
        for _ in range(32):
            try:
                return importlib.import_module(name)
            except ModuleNotFoundError as e:
                if e.name is None or e.name.startswith("sglang_omni"):
                    raise
                mod = _Placeholder(e.name)
                mod.__spec__ = importlib.machinery.ModuleSpec(e.name, None)
                mod.__path__ = []
                sys.modules[e.name] = mod
                for k in [k for k in sys.modules if k.startswith("sglang_omni.")]:
                    del sys.modules[k]
        raise ImportError(name)

    jobs = [("sglang_omni.models.qwen3_omni.config", "Qwen3OmniPipelineConfig", "qwen3_omni_text"),
            ("sglang_omni.models.qwen3_omni.config", "Qwen3OmniSpeechPipelineConfig", "qwen3_omni_speech"),
            ("sglang_omni.models.fishaudio_s2_pro.config", "EntryClass", "s2pro"),
            ("sglang_omni.models.ming_omni.config", "EntryClass", "ming_omni")]
    for module, cls, out in jobs:
        cfg = getattr(load(module), cls)(model_path="/models/checkpoint")
        with open(f"{sys.argv[3]}/{out}.yaml", "w") as f:
            yaml.dump(cfg.model_dump(mode="json"), f, sort_keys=False, default_flow_style=False, indent=2,
                      allow_unicode=True)
    print("exported")
""")

EXPECTED = {
    "qwen3_omni_text": ("Qwen3OmniPipelineConfig",
                        ["preprocessing", "image_encoder", "audio_encoder", "mm_aggregate", "thinker", "decode"]),
    "qwen3_omni_speech": ("Qwen3OmniSpeechPipelineConfig",
                          ["preprocessing", "image_encoder", "audio_encoder", "mm_aggregate", "thinker", "decode",
                           "talker_ar", "code_predictor", "code2wav"]),
    "s2pro": ("S2ProPipelineConfig", ["preprocessing", "tts_engine", "vocoder"]),
    "ming_omni": ("MingOmniPipelineConfig", ["preprocessing", "audio_encoder", "mm_aggregate", "thinker", "decode"]),
}


@pytest.fixture(scope="module")
def exported(tmp_path_factory):
    if not os.path.isdir(os.path.join(REF, "sglang_omni")):
        pytest.skip("the reference is not installed under baseline/_ref")
    out = tmp_path_factory.mktemp("reference_export")
    r = subprocess.run([sys.executable, "-c", EXPORT, ROOT, REF, str(out)], capture_output=True, text=True,
                       timeout=600, cwd=str(out))
    assert r.returncode == 0 and "exported" in r.stdout, r.stderr[-3000:]
    return out


@pytest.mark.parametrize("name", sorted(EXPECTED))
def test_reference_export_loads_and_resolves(exported, name):
    from sglang_omni_b200.config.manager import ConfigManager
    from sglang_omni_b200.utils.misc import import_string

    cfg = ConfigManager.from_file(str(exported / f"{name}.yaml"))
    cls, stages = EXPECTED[name]
    assert type(cfg).__name__ == cls
    assert [s.name for s in cfg.stages] == stages
    for s in cfg.stages:
        assert s.executor.factory.startswith("sglang_omni.")     # the reference's own paths, unedited
        for path in [s.executor.factory, s.get_next] + ([s.input_handler.merge_fn] if s.input_handler.merge_fn else []):
            obj = import_string(path)
            assert callable(obj) and obj.__module__.startswith("sglang_omni_b200."), path


def test_reference_speech_export_compiles_and_serves(exported):
    """The exported 9-stage speech layout, with CLI-style overrides for CPU and tiny random models."""
    from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
    from sglang_omni_b200.config import PipelineRunner, compile_pipeline
    from sglang_omni_b200.config.manager import ConfigManager
    from test_qwen3_omni_pipeline import TINY

    cfg = ConfigManager.from_file(str(exported / "qwen3_omni_speech.yaml"))
    tiny = {k: {a: ("float32" if a == "dtype" else b) for a, b in v.items()} for k, v in TINY.items()}
    idx = {s.name: i for i, s in enumerate(cfg.stages)}
    cli = ["--model_path", "random"]
    for name in ("preprocessing", "image_encoder", "audio_encoder", "thinker", "talker_ar", "code2wav"):
        if name != "preprocessing":
            cli += [f"--stages.{idx[name]}.executor.args.device", "cpu"]
    for i, s in enumerate(cfg.stages):
        if s.relay.device != "cpu":
            cli += [f"--stages.{i}.relay.device", "cpu"]
    cli += [f"--stages.{idx['thinker']}.executor.args.max_batch", "4",
            f"--stages.{idx['thinker']}.executor.args.thinker_max_seq_len", "1024",
            f"--stages.{idx['talker_ar']}.executor.args.max_streams", "4",
            f"--stages.{idx['talker_ar']}.executor.args.talker_max_seq_len", "1024",
            f"--stages.{idx['talker_ar']}.executor.args.tail_frames", "12"]
    overrides = ConfigManager.parse_extra_args(cli)
    for name in ("preprocessing", "image_encoder", "audio_encoder", "thinker", "talker_ar", "code2wav"):
        overrides[f"stages.{idx[name]}.executor.args.overrides"] = tiny
    cfg = ConfigManager.merge_config(cfg, overrides)
    assert cfg.model_path == "random" and cfg.stages[idx["thinker"]].executor.args["speech_enabled"] is True

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            audio = (np.random.default_rng(3).standard_normal(16000) * 0.1).astype(np.float32)
            req = GenerateRequest(prompt="hi", audios=[audio], max_tokens=4,
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True),
                                  output_modalities=["text", "audio"], stream=True)
            text, n_audio, final = [], 0, None
            async for ch in Client(coord).generate(req):
                if ch.finish_reason is not None:
                    final = ch
                elif ch.modality == "audio":
                    n_audio += 1
                elif ch.token_ids:
                    text += ch.token_ids
            assert len(text) == 4 and n_audio > 0 and final is not None

    asyncio.run(main())
