"""vLLM's own engine serving a model through the OSCAR plugin (the drop-in path of the
reference's plugin.py -> backend.py -> metadata.py on vLLM's CUDA worker): a tiny
random-weight decoder with the reference's attention geometry per rank generalised to
24 query / 4 KV heads of D = 256, engine block size 768, three prompts of 700-1500
tokens and 24 greedy tokens each.  Eager mode and with CUDA graphs captured for decode
(vLLM builds the graphs under the dummy scope and replays them with new metadata).
Each engine runs in its own process (tests/vllm_engine_run.py)."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _env():
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT) + os.pathsep + env.get("PYTHONPATH", "")
    return env


def run_engine(mode, oscar=1, *extra):
    out = subprocess.run([sys.executable, str(ROOT / "tests" / "vllm_engine_run.py"), "--mode", mode, "--oscar",
                          str(oscar), *extra], env=_env(), capture_output=True, text=True, timeout=900,
                         cwd=str(ROOT))
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert out.returncode == 0 and lines, out.stderr[-4000:]
    return json.loads(lines[-1])


@pytest.mark.parametrize("mode", ["eager", "graphs"])
def test_vllm_engine_generates_through_oscar(cuda_lib, mode):
    r = run_engine(mode)
    assert r["impls"] == ["oscar_new_b200.backend.OscarAttentionImpl"], r["impls"]
    assert r["last_history_kernel"] in (1, 2, 3)  # a history kernel ran inside the engine
    assert r["repeat_equal"]
    assert [len(t) for t in r["tokens"]] == [24, 24, 24]
    assert all(0 <= x < 2048 for t in r["tokens"] for x in t)


def test_first_token_matches_the_native_backend(cuda_lib):
    """The first generated token comes from the prefill forward, which OSCAR runs through
    the tcgen05 prefill kernel over the exact BF16 current K/V while it writes the
    INT2 history and the window: it must equal the native backend's.  Later tokens read
    the INT2 history and may differ (a random-weight model has nearly flat logits)."""
    native = run_engine("eager", oscar=0)
    assert native["impls"] and "Oscar" not in native["impls"][0]
    oscar = run_engine("eager", oscar=1)
    assert [t[0] for t in oscar["tokens"]] == [t[0] for t in native["tokens"]]


def test_calibrate_on_the_engine_then_serve_with_the_published_rotations(cuda_lib, tmp_path):
    """The calibration driver (reference calibrate.py on vLLM's CUDA worker): native
    attention observed by the worker extension over 1024 synthetic tokens, both passes,
    the device eigensolver, and k_rotation.pt / v_rotation.pt published for both layers;
    then the engine serves through OSCAR with those rotations."""
    import torch

    from oscar_new_b200.rotations import get_rotation, load_checkpoint

    model, out = tmp_path / "model", tmp_path / "rotations"
    run = subprocess.run([sys.executable, str(ROOT / "tests" / "vllm_engine_run.py"), "--make-only",
                          "--model-dir", str(model)], env=_env(), capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-3000:]
    run = subprocess.run([sys.executable, "-m", "oscar_new_b200.calibrate", "--model", str(model), "--output-dir",
                          str(out), "--model-fingerprint", "tiny-qwen3", "--profile-fingerprint", "test",
                          "--synthetic-prompts", "2", "--tokens", "1024", "--max-sweeps", "12", "--memory", "0.25"],
                         env=_env(), capture_output=True, text=True, timeout=900, cwd=str(ROOT))
    assert run.returncode == 0, run.stderr[-4000:]
    for kind in ("k", "v"):
        raw = torch.load(out / f"{kind}_rotation.pt", weights_only=False)
        assert raw["calibration"]["model_fingerprint"] == "tiny-qwen3"
        assert raw["calibration"]["prompt_tokens"] == 1024
        assert sorted(raw["layers"]) == [0, 1]
        for layer in (0, 1):
            ev = raw["layers"][layer]["eigenvalues"]
            assert bool((ev[1:] >= ev[:-1]).all()) and bool((ev > 0).all())
        f = load_checkpoint(str(out / f"{kind}_rotation.pt"))
        assert not f.problems
        r = get_rotation(str(out / f"{kind}_rotation.pt"), "model.layers.1.self_attn.attn", "cpu").float()
        assert float((r.T @ r - torch.eye(256)).abs().max()) < 0.015
    r = run_engine("eager", 1, "--model-dir", str(model), "--rotations", str(out))
    assert r["impls"] == ["oscar_new_b200.backend.OscarAttentionImpl"]
    assert r["last_history_kernel"] in (1, 2, 3)
