"""Host logic of the calibration driver (oscar_new_b200/calibrate.py): which layers are
calibrated, how the token budget becomes prompts, and argument rules."""

import json

import pytest

from oscar_new_b200 import calibrate


def test_full_attention_layers_from_config(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"num_hidden_layers": 3, "head_dim": 256}))
    assert calibrate.full_attention_layers(tmp_path) == [0, 1, 2]
    hybrid = {"text_config": {"head_dim": 256, "layer_types": ["linear_attention", "full_attention"] * 4}}
    (tmp_path / "config.json").write_text(json.dumps(hybrid))
    assert calibrate.full_attention_layers(tmp_path) == [1, 3, 5, 7]
    (tmp_path / "config.json").write_text(json.dumps({"num_hidden_layers": 2, "head_dim": 128}))
    with pytest.raises(ValueError, match="head_dim"):
        calibrate.full_attention_layers(tmp_path)


def test_prompts_hold_exactly_the_budget(tmp_path):
    p = calibrate.build_prompts(1025, synthetic=4, vocab=50)
    assert sum(len(x["prompt_token_ids"]) for x in p) == 1025 and len(p) == 4
    assert all(0 <= t < 50 for x in p for t in x["prompt_token_ids"])
    assert p == calibrate.build_prompts(1025, synthetic=4, vocab=50)  # seeded

    class Tok:
        def encode(self, text):
            return [len(w) for w in text.split()]

    (tmp_path / "d.jsonl").write_text("\n".join(json.dumps({"text": "a bb ccc " * n}) for n in (2, 5)))
    p = calibrate.build_prompts(10, str(tmp_path / "d.jsonl"), Tok())
    assert [x["prompt_token_ids"] for x in p] == [[1, 2, 3, 1, 2, 3], [1, 2, 3, 1]]
    (tmp_path / "d.txt").write_text("\n\n")
    with pytest.raises(ValueError, match="no tokens"):
        calibrate.build_prompts(10, str(tmp_path / "d.txt"), Tok())


def test_argument_rules():
    base = ["--model", "m", "--output-dir", "o", "--model-fingerprint", "f", "--profile-fingerprint", "p"]
    with pytest.raises(ValueError, match="exactly one"):
        calibrate.main(base + ["--tokens", "1024"])
    with pytest.raises(ValueError, match="256..8192"):
        calibrate.main(base + ["--synthetic-prompts", "1", "--tokens", "100"])
