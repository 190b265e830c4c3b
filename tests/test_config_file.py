"""Deployment configuration from one YAML/JSON file: typed sections, loud
errors for unknown fields or wrong types, and the scheduling section written
as the SCHED_* wire format that round-trips through the plugin's reader."""
import json

import pytest

from sched_pass_b200.engine.config_file import apply_sched_env, load_config
from sched_pass_b200.engine.plugin import SchedPluginConfig


def test_yaml_and_json_round_trip(tmp_path):
    y = tmp_path / "c.yaml"
    y.write_text("engine:\n  max_batch: 64\n  prefix_cache: true\nsched:\n  enforce: false\n  timer_every: 4\n"
                 "  clc: off\n")
    ecfg, scfg = load_config(str(y))
    assert ecfg.max_batch == 64 and ecfg.prefix_cache and not scfg.enforce and scfg.timer_every == 4
    env = {}
    wire = apply_sched_env(scfg, env)
    assert env == wire and env["SCHED_ENFORCE"] == "0" and env["SCHED_TIMER_EVERY"] == "4"
    assert SchedPluginConfig.from_env(env) == scfg
    j = tmp_path / "c.json"
    j.write_text(json.dumps({"engine": {"max_context": 8192}}))
    ecfg, scfg = load_config(str(j))
    assert ecfg.max_context == 8192 and scfg == SchedPluginConfig()


@pytest.mark.parametrize("text,msg", [
    ("engine:\n  max_batchh: 3\n", "unknown field"),
    ("engines:\n  max_batch: 3\n", "unknown section"),
    ("engine:\n  prefix_cache: 1\n", "true/false"),
    ("engine:\n  max_batch: big\n", "integer"),
    ("sched:\n  clc: sometimes\n", "off|on|auto"),
])
def test_bad_files_are_refused(tmp_path, text, msg):
    p = tmp_path / "bad.yaml"
    p.write_text(text)
    with pytest.raises(ValueError, match=msg):
        load_config(str(p))
