"""Calibration driver: serve the native BF16 model in vLLM, run the two calibration
passes over a token budget, publish the K/V rotation pair, exit.

Same flow as the reference's ``oscar_ascend/calibrate.py:11-113`` on vLLM's CUDA
worker: the engine runs with native attention (OSCAR disabled) and the worker
extension ``oscar_new_b200.calibration_worker.CalibrationWorkerExtension``;
``oscar_calibration_begin(layers, budget)``, pass 1 (query Grams), ``..._second_pass``,
pass 2 (SST-weighted value Grams), ``..._finish(output_dir, provenance, sweeps)``; rank 0
publishes ``k_rotation.pt`` / ``v_rotation.pt`` and exactly one rank must report it.

Prompts: ``--data`` names a text file (one prompt per line) or a JSONL file (a "text"
field per record) that the model's tokenizer turns into at most ``--tokens`` tokens;
``--synthetic-prompts N`` instead draws N seeded random token-id prompts over the same
budget, for models served without a tokenizer (tests, smoke runs).

    python -m oscar_new_b200.calibrate --model DIR --output-dir OUT \\
        --model-fingerprint F --profile-fingerprint P (--data FILE | --synthetic-prompts N)
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import uuid
from pathlib import Path


def full_attention_layers(model_dir) -> list:
    """Indices of the FULL attention layers from the model's config.json: its
    ``layer_types`` when present (hybrid models), else every layer."""
    cfg = json.loads((Path(model_dir) / "config.json").read_text())
    cfg = cfg.get("text_config", cfg)
    if cfg.get("head_dim", 256) != 256:
        raise ValueError(f"OSCAR calibrates head_dim 256 attention; the model has {cfg.get('head_dim')}")
    types = cfg.get("layer_types")
    if types is None:
        return list(range(int(cfg["num_hidden_layers"])))
    full = [i for i, t in enumerate(types) if t == "full_attention"]
    if not full:
        raise ValueError("the model has no full-attention layer")
    return full


def _texts(path):
    p = Path(path)
    lines = [ln for ln in p.read_text().splitlines() if ln.strip()]
    if p.suffix == ".jsonl":
        return [json.loads(ln)["text"] for ln in lines]
    return lines


def build_prompts(budget, data=None, tokenizer=None, synthetic=0, vocab=None, seed=0):
    """Token-id prompts holding `budget` tokens in total."""
    import torch

    if synthetic:
        g = torch.Generator().manual_seed(seed)
        sizes = [budget // synthetic + (1 if i < budget % synthetic else 0) for i in range(synthetic)]
        return [{"prompt_token_ids": torch.randint(0, vocab, (n,), generator=g).tolist()} for n in sizes if n]
    prompts, left = [], budget
    for text in _texts(data):
        ids = tokenizer.encode(text)[:left]
        if ids:
            prompts.append({"prompt_token_ids": ids})
            left -= len(ids)
        if left == 0:
            break
    if not prompts:
        raise ValueError("the calibration data holds no tokens")
    return prompts


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", required=True)
    ap.add_argument("--output-dir", type=Path, required=True)
    ap.add_argument("--model-fingerprint", required=True)
    ap.add_argument("--profile-fingerprint", required=True)
    ap.add_argument("--data", default=os.getenv("OSCAR_CALIBRATION_DATA"))
    ap.add_argument("--synthetic-prompts", type=int, default=0)
    ap.add_argument("--tokens", type=int, default=int(os.getenv("OSCAR_CALIBRATION_TOKENS", "1024")))
    ap.add_argument("--max-sweeps", type=int, default=int(os.getenv("OSCAR_CALIBRATION_SWEEPS", "12")))
    ap.add_argument("--tensor-parallel-size", type=int, default=1)
    ap.add_argument("--memory", type=float, default=float(os.getenv("OSCAR_CALIBRATION_MEMORY", "0.75")))
    args = ap.parse_args(argv)
    if not 256 <= args.tokens <= 8192 or not 2 <= args.max_sweeps <= 32:
        raise ValueError("calibration tokens must be 256..8192 and Jacobi sweeps 2..32")
    if bool(args.data) == bool(args.synthetic_prompts):
        raise ValueError("give exactly one of --data and --synthetic-prompts")
    # native attention while calibrating; vLLM is imported only after this is set
    os.environ["OSCAR_ENABLED"] = "0"
    os.environ["OSCAR_ASCEND_ENABLED"] = "0"
    os.environ["OSCAR_CALIBRATING"] = "1"
    from vllm import LLM, SamplingParams

    layers = full_attention_layers(args.model)
    cfg = json.loads((Path(args.model) / "config.json").read_text())
    llm = LLM(
        model=args.model,
        tensor_parallel_size=args.tensor_parallel_size,
        worker_extension_cls="oscar_new_b200.calibration_worker.CalibrationWorkerExtension",
        dtype="bfloat16",
        enforce_eager=True,
        enable_prefix_caching=False,
        max_model_len=max(4096, args.tokens + 1),
        max_num_batched_tokens=min(2048, args.tokens),
        max_num_seqs=1,
        gpu_memory_utilization=args.memory,
        compilation_config={"mode": 0, "cudagraph_mode": "NONE"},
        skip_tokenizer_init=bool(args.synthetic_prompts),
    )
    try:
        tokenizer = None if args.synthetic_prompts else llm.get_tokenizer()
        prompts = build_prompts(args.tokens, args.data, tokenizer, args.synthetic_prompts,
                                cfg.get("text_config", cfg).get("vocab_size"))
        budget = sum(len(p["prompt_token_ids"]) for p in prompts)
        sampling = SamplingParams(temperature=0, max_tokens=1, ignore_eos=True, seed=0, detokenize=False)
        provenance = {
            "model_fingerprint": args.model_fingerprint,
            "data_source": args.data or f"synthetic:{args.synthetic_prompts}",
            "profile_fingerprint": args.profile_fingerprint,
            "run_id": uuid.uuid4().hex,
            "prompt_sha256": hashlib.sha256(json.dumps(prompts, sort_keys=True).encode()).hexdigest(),
            "prompt_tokens": budget,
            "generator_version": 1,
        }
        llm.collective_rpc("oscar_calibration_begin", args=(layers, budget))
        print("[OSCAR calibration] pass 1/2: query covariances", flush=True)
        llm.generate(prompts, sampling, use_tqdm=False)
        llm.collective_rpc("oscar_calibration_second_pass")
        print("[OSCAR calibration] pass 2/2: SST-weighted value covariances", flush=True)
        llm.generate(prompts, sampling, use_tqdm=False)
        results = llm.collective_rpc("oscar_calibration_finish",
                                     args=(str(args.output_dir), provenance, args.max_sweeps))
        if sum(bool(r.get("published")) for r in results) != 1:
            raise RuntimeError("calibration did not publish exactly one K/V rotation pair")
        print(f"[OSCAR calibration] K/V rotations written to {args.output_dir}", flush=True)
        return results
    finally:
        shutdown = getattr(getattr(llm.llm_engine, "engine_core", None), "shutdown", None)
        if shutdown is not None:
            shutdown()


if __name__ == "__main__":
    main()
