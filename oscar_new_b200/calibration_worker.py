"""Calibration passes run inside native-attention workers (one process per GPU).

Same RPC flow as the reference's ``oscar_ascend/calibration_worker.py:14-180``:
``begin`` installs an observe hook on vLLM's native CUDA attention
(``FlashAttentionImpl.forward``), pass 1 accumulates the query Gram ``sum q^T q`` per
layer, ``second_pass`` normalises it to ``Cq = sum / (N*G)``, pass 2 accumulates the
SST-weighted value Gram ``sum w v^T v`` with ``w = max(k Cq k^T, 0)``, and ``finish``
sums the covariance stack over ranks with one all-reduce, rank 0 solves the batched
Jacobi eigenproblems on the device and atomically writes ``k_rotation.pt`` /
``v_rotation.pt`` (format version 1, ``source_grouping`` "layer").

Generalised over the reference's fixed TP4 geometry (Hq=6, Hkv=1 per rank):

* each rank may hold any number of KV heads ``Hl`` with ``G = Hq/Hkv`` query heads each;
  per-head statistics are kept and the published matrix of a layer is the mean of the
  per-head covariances over all KV heads of all ranks (the reference's ``/4``);
* ``shard="heads"`` (the reference's TP case): ranks own distinct heads and see every
  token, so Cq is rank-local and only ``finish`` communicates;
* ``shard="tokens"``: ranks own distinct token segments for every head, so
  ``second_pass`` all-reduces the query sums and counts before Cq exists (a real
  exchange step: the SST weights need the global Cq), and ``finish`` all-reduces the
  value sums and weight totals.

The arithmetic goes through ``ops`` (default: the CUDA calibration kernels, which fail
on non-CUDA tensors).  Tests on CPU pass a different ``ops``/``eigensolver``.
"""

from __future__ import annotations

import functools
import os
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import torch

DIM = 256
_installed = False
_session: "CalibrationSession | None" = None


def _default_group():
    """vLLM's tensor-parallel device group when running under vLLM, else the default group."""
    import torch.distributed as dist

    try:
        from vllm.distributed import get_tp_group

        return get_tp_group().device_group
    except Exception:  # noqa: BLE001 - outside a vLLM worker
        return None if not (dist.is_available() and dist.is_initialized()) else dist.group.WORLD


class CalibrationSession:
    """Per-process calibration state for the layers this process observes."""

    def __init__(self, layers, token_budget, device, num_kv_heads, group_size, shard="heads", group=None, ops=None):
        if shard not in ("heads", "tokens"):
            raise ValueError("shard must be 'heads' or 'tokens'")
        if num_kv_heads <= 0 or group_size <= 0:
            raise ValueError("calibration needs at least one KV head and one query head per KV head")
        if ops is None:
            from . import calibration_kernels as ops
        self.ops = ops
        self.shard = shard
        self.group = group
        self.budget = int(token_budget)
        self.heads = int(num_kv_heads)
        self.group_size = int(group_size)
        self.device = torch.device(device)
        self.phase = 1
        self.states = {
            int(layer): {
                "q_sum": torch.zeros((self.heads, DIM, DIM), dtype=torch.float32, device=self.device),
                "v_sum": torch.zeros((self.heads, DIM, DIM), dtype=torch.float32, device=self.device),
                "weight_sum": torch.zeros((self.heads,), dtype=torch.float32, device=self.device),
                "q_tokens": 0,
                "v_tokens": 0,
            }
            for layer in layers
        }

    # --- collectives ----------------------------------------------------------
    def _world(self):
        import torch.distributed as dist

        if self.group is None or not dist.is_initialized():
            return 1, 0
        return dist.get_world_size(self.group), dist.get_rank(self.group)

    def _all_reduce(self, tensor):
        import torch.distributed as dist

        if self._world()[0] > 1:
            dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=self.group)
        return tensor

    # --- passes ---------------------------------------------------------------
    def observe(self, layer_index, query, key, value, num_tokens):
        """Accumulate the current tokens of one layer (reference calibration_worker.py:53-83)."""
        state = self.states.get(int(layer_index))
        if state is None or self.phase == 0:
            return
        counter = "q_tokens" if self.phase == 1 else "v_tokens"
        limit = self.budget if self.phase == 1 else state["q_tokens"]
        take = int(min(int(num_tokens), query.shape[0], limit - state[counter]))
        if take <= 0:
            return
        h, g = self.heads, self.group_size
        if self.phase == 1:
            # one launch: KV head j accumulates its G query heads into q_sum[j]
            self.ops.accumulate_gram_grouped(query[:take].reshape(take, h * g, DIM), state["q_sum"])
        else:
            k = key[:take].reshape(take, h, DIM)
            v = value[:take].reshape(take, h, DIM)
            prepared = state.get("q_cov_sst")
            if prepared is None:
                w = self.ops.sst_weights_per_head(k, state["q_cov"], state["weight_sum"])
            else:
                w = self.ops.sst_weights_per_head(k, state["q_cov"], state["weight_sum"], prepared=prepared)
            self.ops.accumulate_gram_grouped(v, state["v_sum"], w)
        state[counter] += take

    def second_pass(self):
        """Normalise the query Grams (reference calibration_worker.py:108-118)."""
        if self.phase != 1:
            raise RuntimeError("second_pass follows the first calibration pass")
        layers = sorted(self.states)
        if self.shard == "tokens":
            counts = torch.tensor([self.states[i]["q_tokens"] for i in layers], dtype=torch.float64,
                                  device=self.device)
            self._all_reduce(counts)
            stack = torch.stack([self.states[i]["q_sum"] for i in layers])
            self._all_reduce(stack)
            for j, i in enumerate(layers):
                self.states[i]["q_sum"] = stack[j]
                self.states[i]["q_tokens_total"] = int(counts[j].item())
        else:
            for i in layers:
                self.states[i]["q_tokens_total"] = self.states[i]["q_tokens"]
        totals = {i: self.states[i]["q_tokens_total"] for i in layers}
        if not totals or min(totals.values()) < DIM:
            raise RuntimeError(f"Insufficient real-model Q samples; no rotations generated: {totals}")
        # operators that keep a prepared form of the query covariances (the tensor-core
        # SST kernel's exact bf16 split) build it here, once for the whole second pass
        prepare = getattr(self.ops, "prepare_sst_covariances", None)
        for state in self.states.values():
            state["q_cov"] = self.ops.normalize(state["q_sum"], state["q_tokens_total"] * self.group_size)
            if prepare is not None:
                state["q_cov_sst"] = prepare(state["q_cov"])
        self.phase = 2
        return {"phase": 2, "tokens_per_layer": {i: s["q_tokens"] for i, s in self.states.items()}}

    def covariances(self):
        """The per-layer ``[Cq_layer, Cv_layer]`` stack, identical on every rank."""
        layers = sorted(self.states)
        for i in layers:
            s = self.states[i]
            if s["v_tokens"] != s["q_tokens"] or s.get("q_tokens_total", 0) < DIM:
                raise RuntimeError(f"Calibration pass sample mismatch at layer {i}")
        if self.shard == "tokens":
            weights = self._all_reduce(torch.stack([self.states[i]["weight_sum"] for i in layers]))
            vsum = self._all_reduce(torch.stack([self.states[i]["v_sum"] for i in layers]))
        else:
            weights = torch.stack([self.states[i]["weight_sum"] for i in layers])
            vsum = torch.stack([self.states[i]["v_sum"] for i in layers])
        # startup-only scalar check; no activations leave the device
        if not bool(torch.isfinite(weights).all()) or not bool((weights > 0).all()):
            raise RuntimeError("Degenerate SST weights")
        # per layer: Cq = sum over KV heads of the normalised query Grams, Cv = sum over
        # KV heads of v_sum / max(weight_sum, 1e-30); all layers at once, stacked as
        # [Cq_0, Cv_0, Cq_1, Cv_1, ...]
        q = torch.stack([self.states[i]["q_cov"] for i in layers]).sum(1)
        v = (vsum / weights.clamp_min(1e-30)[:, :, None, None]).sum(1)
        stack = torch.stack((q, v), 1).reshape(2 * len(layers), DIM, DIM)
        world, _ = self._world()
        if self.shard == "heads":
            self._all_reduce(stack)
            total_heads = self.heads * world
        else:
            total_heads = self.heads
        return self.ops.normalize(stack, total_heads)

    def finish(self, output_dir, provenance, max_sweeps, eigensolver=None):
        """All-reduce, rank-0 eigensolve and atomic publication (reference :121-180)."""
        self.phase = 0
        covariances = self.covariances()
        world, rank = self._world()
        if rank != 0:
            return {"rank": rank, "published": False}
        if eigensolver is None:
            eigensolver = self.ops.calibrated_rotations
        rotations, eigenvalues, convergence = eigensolver(covariances, max_sweeps=max_sweeps)
        # the reference's per-matrix check, allclose(R^T R, I, atol=rtol=0.005) and finite
        # entries, batched where the rotations are (one launch instead of 2 x layers host
        # matrix products)
        gram = torch.matmul(rotations.transpose(-1, -2), rotations)
        eye = torch.eye(DIM, dtype=rotations.dtype, device=rotations.device)
        valid = (torch.isfinite(rotations).flatten(1).all(1)
                 & ((gram - eye).abs() <= 0.005 + 0.005 * eye).flatten(1).all(1))
        rotations_cpu, eigenvalues_cpu, valid = _to_host(rotations, eigenvalues, valid)
        output = Path(output_dir)
        output.mkdir(parents=True, exist_ok=True)
        layers = sorted(self.states)
        files = []
        for kind, offset, objective in (("k", 0, "qqt_r_h_pbr"), ("v", 1, "sst_r_h_pbr")):
            result = {
                "format_version": 1,
                "source_grouping": "layer",
                "objective": objective,
                "model_fingerprint": provenance.get("model_fingerprint", ""),
                "calibration": {
                    **provenance,
                    **convergence,
                    "arithmetic": "cuda_sm100a",
                    "shard": self.shard,
                    "world_size": world,
                    "tokens_per_layer": {i: self.states[i]["q_tokens_total"] for i in layers},
                },
                "layers": {},
            }
            for number, index in enumerate(layers):
                # a copy of its own: a view would make the file carry the whole K + V stack
                matrix = rotations_cpu[number * 2 + offset].clone()
                if not bool(valid[number * 2 + offset]):
                    raise RuntimeError(f"Generated {kind} rotation for layer {index} failed validation")
                result["layers"][index] = {"layer_id": index, "rotation": matrix,
                                           "eigenvalues": eigenvalues_cpu[number * 2 + offset].clone()}
            files.append((result, output / f"{kind}_rotation.pt"))
        # both files are validated; write them side by side (serialisation and the zip
        # checksums release the interpreter lock) and publish each by an atomic rename
        with ThreadPoolExecutor(max_workers=len(files)) as pool:
            for done in [pool.submit(_publish, result, path) for result, path in files]:
                done.result()
        return {"rank": 0, "published": True, **convergence}


def _to_host(*tensors):
    """Device tensors to host copies through pinned buffers, one synchronisation."""
    if not tensors[0].is_cuda:
        return tuple(t.cpu() for t in tensors)
    host = tuple(torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in tensors)
    for h, t in zip(host, tensors):
        h.copy_(t, non_blocking=True)
    torch.cuda.current_stream(tensors[0].device).synchronize()
    return host


def _publish(result, path):
    temporary = path.with_suffix(".pt.tmp")
    torch.save(result, temporary)
    os.replace(temporary, path)


# --- vLLM worker extension (reference calibration_worker.py:14-50) --------------------


class CalibrationWorkerExtension:
    """Named RPCs for ``LLM(worker_extension_cls=...)`` + ``collective_rpc``."""

    def oscar_calibration_begin(self, layers, token_budget):
        return begin(self, layers, token_budget)

    def oscar_calibration_second_pass(self):
        return second_pass(self)

    def oscar_calibration_finish(self, output_dir, provenance, max_sweeps):
        return finish(self, output_dir, provenance, max_sweeps)


# Native attention implementations vLLM may pick on a CUDA worker (FlashInfer on B200,
# FlashAttention elsewhere); calibration observes whichever ones the engine loaded.
NATIVE_IMPLS = (("vllm.v1.attention.backends.flash_attn", "FlashAttentionImpl"),
                ("vllm.v1.attention.backends.flashinfer", "FlashInferImpl"))


def install_hook(impl_cls=None):
    """Wrap the native attention implementations' ``forward`` to observe Q/K/V."""
    global _installed
    if _installed:
        return
    if impl_cls is not None:
        classes = [impl_cls]
    else:
        classes = []
        for module_name, name in NATIVE_IMPLS:
            module = sys.modules.get(module_name)
            if module is None or getattr(getattr(module, "__spec__", None), "_initializing", False):
                continue
            if getattr(module, name, None) is not None:
                classes.append(getattr(module, name))
        if not classes:
            raise RuntimeError("Native attention must be initialized before calibration begin RPC")
    for cls in classes:
        original = cls.forward

        def make(original):
            @functools.wraps(original)
            def forward(impl, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs):
                result = original(impl, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs)
                if _session is not None and _session.phase and attn_metadata is not None and key is not None \
                        and value is not None:
                    observe(impl, layer, query, key, value, attn_metadata.num_actual_tokens)
                return result
            return forward

        cls.forward = make(original)
    _installed = True


def observe(impl, layer, query, key, value, num_tokens):
    from .plugin import is_draft_layer
    from .rotations import layer_index

    if _session is None or is_draft_layer(layer.layer_name) or impl.head_size != DIM:
        return
    if str(getattr(impl, "attn_type", "decoder")).split(".")[-1].lower() != "decoder":
        return
    if impl.num_kv_heads != _session.heads or impl.num_heads != _session.heads * _session.group_size:
        raise ValueError("calibration geometry changed between layers")
    if not query.is_cuda:
        raise ValueError("Calibration Q/K/V must stay on the GPU")
    _session.observe(layer_index(layer.layer_name), query, key, value, num_tokens)


def begin(worker, layers, token_budget, num_kv_heads=None, group_size=None):
    """Start pass 1 (reference :86-105).  Geometry defaults to the worker's model config."""
    global _session
    install_hook()
    if num_kv_heads is None or group_size is None:
        mc = worker.model_runner.model_config
        pc = worker.model_runner.parallel_config
        num_kv_heads = mc.get_num_kv_heads(pc)
        group_size = mc.get_num_attention_heads(pc) // num_kv_heads
    device = torch.device("cuda", torch.cuda.current_device())
    _session = CalibrationSession(layers, token_budget, device, num_kv_heads, group_size, "heads", _default_group())
    return {"phase": 1, "layers": len(layers)}


def second_pass(worker):
    if _session is None:
        raise RuntimeError("calibration begin RPC was not called")
    return _session.second_pass()


def finish(worker, output_dir, provenance, max_sweeps):
    global _session
    if _session is None:
        raise RuntimeError("calibration begin RPC was not called")
    try:
        return _session.finish(output_dir, provenance, max_sweeps)
    finally:
        _session = None
