"""Serve a tiny random-weight decoder (head_dim 256, 24 query / 4 KV heads, 2 layers)
with vLLM and the OSCAR plugin, in this process, and print one JSON line.

Used by tests/test_gpu_vllm_engine.py in a subprocess (one engine per process).  No
network: the model is written locally (transformers, seeded random weights), prompts
are token ids (no tokenizer), rotations are the synthetic orthogonal * Hadamard ones.

    python tests/vllm_engine_run.py --mode eager|graphs
"""

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def make_tiny_model(d: Path):
    """Seeded random-weight Qwen3-architecture decoder: 2 layers, hidden 1024, 24 query /
    4 KV heads of D = 256, vocabulary 2048 (written once per directory)."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    if (d / "config.json").exists():
        return
    cfg = Qwen3Config(vocab_size=2048, hidden_size=1024, intermediate_size=2048, num_hidden_layers=2,
                      num_attention_heads=24, num_key_value_heads=4, head_dim=256, max_position_embeddings=8192,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    Qwen3ForCausalLM(cfg).to(torch.bfloat16).save_pretrained(d)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["eager", "graphs"], default="eager")
    ap.add_argument("--oscar", type=int, default=1)
    ap.add_argument("--model-dir", default=None, help="reuse / create the tiny model here")
    ap.add_argument("--make-only", action="store_true", help="write the tiny model and exit")
    ap.add_argument("--rotations", default=None, help="directory with k_rotation.pt / v_rotation.pt")
    args = ap.parse_args()
    os.environ["OSCAR_ENABLED"] = str(args.oscar)
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    import torch

    d = Path(args.model_dir) if args.model_dir else Path(tempfile.mkdtemp(prefix="oscar_tiny_"))
    d.mkdir(parents=True, exist_ok=True)
    make_tiny_model(d)
    if args.make_only:
        return
    from oscar_new_b200.synthetic import rotation

    for name, seed in (("K", 1), ("V", 2)):
        if args.rotations:
            p = Path(args.rotations) / f"{name.lower()}_rotation.pt"
        else:
            p = d / f"{name.lower()}_rotation.pt"
            torch.save({"layers": {i: {"rotation": rotation(seed)} for i in range(2)}}, p)
        os.environ[f"VLLM_OSCAR_{name}_ROTATION_PATH"] = str(p)
    os.environ["VLLM_OSCAR_SINK_TOKENS"] = "4"
    os.environ["VLLM_OSCAR_RECENT_TOKENS"] = "128"
    from oscar_new_b200 import _lib, plugin

    plugin.register()  # what vLLM's general-plugin entry point calls
    from vllm import LLM, SamplingParams

    extra = {"enforce_eager": True} if args.mode == "eager" else {
        "enforce_eager": False, "compilation_config": {"mode": 0, "cudagraph_mode": "FULL_DECODE_ONLY"}}
    llm = LLM(model=str(d), skip_tokenizer_init=True, block_size=768, max_model_len=4096,
              gpu_memory_utilization=0.25, enable_prefix_caching=False, dtype="bfloat16", max_num_seqs=8, seed=0,
              **extra)
    g = torch.Generator().manual_seed(1)
    prompts = [{"prompt_token_ids": torch.randint(0, 2048, (n,), generator=g).tolist()} for n in (1000, 700, 1500)]
    sp = SamplingParams(max_tokens=24, temperature=0.0, detokenize=False)
    first = [list(o.outputs[0].token_ids) for o in llm.generate(prompts, sp)]
    again = [list(o.outputs[0].token_ids) for o in llm.generate(prompts, sp)]
    def impl_names(model):
        return sorted({type(m.impl).__module__ + "." + type(m.impl).__name__
                       for m in model.modules() if getattr(m, "impl", None) is not None})

    impls = set()
    for names in llm.apply_model(impl_names):
        impls.update(names)
    print(json.dumps({"mode": args.mode, "tokens": first, "repeat_equal": first == again,
                      "last_history_kernel": int(_lib.lib().oscar_last_history_kernel()),
                      "impls": sorted(impls)}), flush=True)


if __name__ == "__main__":
    main()
