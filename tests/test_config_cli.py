"""Config schema validation, fusion, dotted overrides, YAML round trip, registry and CLI."""
import subprocess
import sys

import pytest

from sglang_omni_b200.config import ConfigManager, ExecutorConfig, PipelineConfig, StageConfig, StreamTargetConfig
from sglang_omni_b200.models.registry import PIPELINE_CONFIG_REGISTRY
from sglang_omni_b200.models.toy.config import ToyPipelineConfig
from sglang_omni_b200.utils.misc import import_string


def _stage(name, nxt="sglang_omni_b200.models.common.text_stages.terminal"):
    return StageConfig(name=name, executor=ExecutorConfig(factory="x.y"), get_next=nxt)


def test_validation_errors():
    with pytest.raises(ValueError):
        PipelineConfig(model_path="m", entry_stage="a", stages=[_stage("a"), _stage("a")])
    with pytest.raises(ValueError):
        PipelineConfig(model_path="m", entry_stage="zz", stages=[_stage("a")])
    with pytest.raises(ValueError):
        PipelineConfig(model_path="m", entry_stage="a", stages=[_stage("a"), _stage("b"), _stage("c")],
                       fused_stages=[["a", "c"]])


def test_fusion_collapses_adjacent_group():
    cfg = PipelineConfig(model_path="m", entry_stage="a", stages=[_stage("a"), _stage("b"), _stage("c")],
                         fused_stages=[["a", "b"]])
    stages, name_map, entry = cfg.apply_fusion()
    assert [s.name for s in stages] == ["b", "c"]
    assert entry == "b" and name_map["a"] == "b"
    assert stages[0].executor.factory.endswith("build_fused_executor")


def test_overrides_and_yaml_roundtrip(tmp_path):
    cfg = ToyPipelineConfig()
    extra = ConfigManager.parse_extra_args(["--stages.1.executor.args.max_batch", "4", "--name=toy2",
                                            "--endpoints.base_port", "17000"])
    cfg2 = ConfigManager.merge_config(cfg, extra)
    assert cfg2.stages[1].executor.args["max_batch"] == 4 and cfg2.name == "toy2"
    p = tmp_path / "c.yaml"
    ConfigManager.to_file(cfg2, str(p))
    cfg3 = ConfigManager.from_file(str(p))
    assert type(cfg3).__name__ == "ToyPipelineConfig" and cfg3.model_dump() == cfg2.model_dump()


def test_registry_and_reference_paths():
    assert PIPELINE_CONFIG_REGISTRY.get_config("ToyLlamaForCausalLM") is ToyPipelineConfig
    # factory paths written for the reference package resolve to this package
    assert import_string("sglang_omni.models.toy.config.to_decoder") is \
        import_string("sglang_omni_b200.models.toy.config.to_decoder")


def test_cli_config_view(tmp_path):
    cfg = ToyPipelineConfig()
    p = tmp_path / "toy.yaml"
    ConfigManager.to_file(cfg, str(p))
    out = subprocess.run([sys.executable, "-m", "sglang_omni_b200.cli", "config", "view", "--config", str(p)],
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "decoder" in out.stdout


def test_console_script_declared():
    """``sgl-omni`` (the reference's command name) is a console script of the package."""
    import os
    import re

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = open(os.path.join(root, "setup.py")).read()
    assert re.search(r'"sgl-omni=sglang_omni_b200\.cli\.cli:main"', src)
    from sglang_omni_b200.cli.cli import main

    import pytest

    with pytest.raises(SystemExit) as e:
        main(["--help"])
    assert e.value.code == 0


def test_validation_reports_every_problem_at_once():
    bad = _stage("b")
    bad.stream_to = [StreamTargetConfig(to_stage="nowhere")]
    with pytest.raises(ValueError) as e:
        PipelineConfig(model_path="", entry_stage="zz", stages=[_stage("a"), bad, _stage("a")],
                       terminal_stages=["gone"], fused_stages=[["a", "missing"]])
    msg = str(e.value)
    for part in ("two stages are named 'a'", "no model_path", "entry stage 'zz'", "'nowhere' is not a stage",
                 "terminal stage 'gone'", "names a stage that does not exist"):
        assert part in msg, (part, msg)
    ok = PipelineConfig(model_path="m", entry_stage="a", stages=[_stage("a"), _stage("b")])
    assert ok.problems() == []
