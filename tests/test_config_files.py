"""The shipped YAML configurations (nested model schema) build exactly the
named presets."""

import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("name,preset", [("genesis_1b", "genesis-1b"), ("genesis_7b_nvfp4", "genesis-7b-nvfp4"),
                                         ("genesis_40b_moe", "genesis-40b-moe")])
def test_yaml_matches_preset(name, preset):
    from llm_research_b200.models.presets import build_hlrt_config
    from olympus.utils.config import hlrt_config_from_yaml

    got = hlrt_config_from_yaml(os.path.join(ROOT, "genesis", "training", "configs", f"{name}.yaml"))
    want = build_hlrt_config(preset)
    assert got.to_dict() == want.to_dict()
