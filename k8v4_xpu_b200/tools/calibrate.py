"""GPTQ calibration on a live model: input Hessians of every quantized linear.

The reference collects them by installing forward pre-hooks in its vLLM
workers and running calibration prompts through the served model
(``tools/calibrate_swift_bake.py:34-52,121-158``): each hook accumulates
``X^T X`` of its linear's input, row-parallel inputs (sharded along K under
TP) are all-gathered first so every rank sees the full input, every 64th row
is held out of the statistics, and ``hessians.pt`` is written atomically
(``:104-106``). Here the same happens on this framework's own model:

* :class:`Calibrator` swaps each :class:`Int4Linear` of a :class:`DenseModel`
  (and of its MTP layer) for a tapped copy that feeds the linear's input to an
  accumulator before running the GEMM. Fused projections map back to the
  checkpoint's linears: ``qkv_proj`` feeds ``q_proj``, ``k_proj`` and
  ``v_proj`` (one shared input, one Hessian), ``gate_up_proj`` feeds
  ``gate_proj`` and ``up_proj``.
* Int8 inputs of the W4A8 path are dequantized (codes x row scale) first.
* ``o_proj`` and ``down_proj`` are row-parallel: under TP their inputs are
  all-gathered along K across the TP group (every rank calls the collective,
  so every rank must run the same forwards).
* Hessians accumulate on the device in fp32 (``X^T X`` and a row count) and
  leave as ``H = 2 X^T X / n`` in fp64 on the CPU, the form
  ``tools.bake.gptq_quantize`` takes.
* Held-out rows (global row index % ``holdout_every`` == ``holdout_every`` - 1)
  are kept, up to a cap, for :meth:`Calibrator.heldout_error`.

    python -m k8v4_xpu_b200.tools.calibrate --preset tiny --prompts 8 --len 512 --out hessians.pt
    python -m k8v4_xpu_b200.tools.bake dense --src DENSE --out BAKED --hessians hessians.pt
"""
from __future__ import annotations

import argparse
import json
import os
import re

import torch

from ..layers.linear import Int4Linear

# fused projection -> the checkpoint linears that read the same input
_UNFUSED = {
    "self_attn.qkv_proj": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"),
    "mlp.gate_up_proj": ("mlp.gate_proj", "mlp.up_proj"),
    "self_attn.o_proj": ("self_attn.o_proj",),
    "mlp.down_proj": ("mlp.down_proj",),
}
# inputs sharded along K under tensor parallelism
_ROW_PARALLEL = ("self_attn.o_proj", "mlp.down_proj")


def checkpoint_names(fused_name: str) -> tuple[str, ...]:
    """Checkpoint linear names that a fused projection's input calibrates."""
    for suffix, names in _UNFUSED.items():
        if fused_name.endswith(suffix):
            prefix = fused_name[: -len(suffix)]
            return tuple(prefix + n for n in names)
    return (fused_name,)


class _Stat:
    """Running ``X^T X`` (fp32, on the inputs' device) and the row count."""

    def __init__(self, k: int, device):
        self.xtx = torch.zeros((k, k), dtype=torch.float32, device=device)
        self.rows = 0   # rows seen
        self.used = 0   # rows accumulated (the rest are held out)
        self.heldout: list[torch.Tensor] = []
        self.heldout_rows = 0


class _Tapped(Int4Linear):
    """An :class:`Int4Linear` sharing the original's weights, whose calls
    first hand their input to the calibrator."""

    def __init__(self, inner: Int4Linear, calib: "Calibrator"):
        self.__dict__.update(inner.__dict__)
        self._inner = inner
        self._calib = calib

    def __call__(self, x=None, xq=None, xs=None, **kw):
        seen = x if x is not None else xq.float() * xs.float().view(-1, 1)
        self._calib._observe(self.name, seen)
        return type(self._inner).__call__(self._inner, x=x, xq=xq, xs=xs, **kw)


class Calibrator:
    """Collects the input Hessians of a model's quantized linears.

    ``model`` is a :class:`~k8v4_xpu_b200.models.dense.DenseModel` (or any
    object with ``layers`` of ``LayerWeights``, an optional ``mtp`` and a
    ``comm`` / ``tp`` pair). ``select`` is a regex on checkpoint linear names
    (default: all); unselected linears are left untouched.
    """

    def __init__(self, model, select: str | None = None, holdout_every: int = 64, holdout_cap: int = 4096):
        if holdout_every < 2:
            raise ValueError("holdout_every must be at least 2")
        self.model = model
        self.select = re.compile(select) if select else None
        self.holdout_every = int(holdout_every)
        self.holdout_cap = int(holdout_cap)
        self.stats: dict[str, _Stat] = {}
        self._swapped: list[tuple[object, str, Int4Linear]] = []

    # ------------------------------------------------------------ attach
    def _holders(self):
        for L in self.model.layers:
            yield L
        mtp = getattr(self.model, "mtp", None)
        if mtp is not None:
            yield mtp
            yield mtp.layer

    def _wanted(self, fused_name: str) -> bool:
        return self.select is None or any(self.select.search(n) for n in checkpoint_names(fused_name))

    def attach(self) -> "Calibrator":
        if self._swapped:
            raise RuntimeError("calibrator already attached")
        for holder in self._holders():
            for attr, lin in list(vars(holder).items()):
                if isinstance(lin, Int4Linear) and not isinstance(lin, _Tapped) and self._wanted(lin.name):
                    setattr(holder, attr, _Tapped(lin, self))
                    self._swapped.append((holder, attr, lin))
        return self

    def detach(self) -> None:
        for holder, attr, lin in reversed(self._swapped):
            setattr(holder, attr, lin)
        self._swapped.clear()

    def __enter__(self) -> "Calibrator":
        return self.attach()

    def __exit__(self, *exc) -> None:
        self.detach()

    # ----------------------------------------------------------- observe
    def _gather_k(self, name: str, x: torch.Tensor) -> torch.Tensor:
        tp = int(getattr(self.model, "tp", 1))
        if tp > 1 and name.endswith(_ROW_PARALLEL):
            return self.model.comm.all_gather(x.contiguous(), dim=-1)
        return x

    def _observe(self, name: str, x: torch.Tensor) -> None:
        x = self._gather_k(name, x.reshape(-1, x.shape[-1]))
        st = self.stats.get(name)
        if st is None:
            st = self.stats[name] = _Stat(x.shape[-1], x.device)
        n = x.shape[0]
        idx = torch.arange(st.rows, st.rows + n, device=x.device)
        hold = (idx % self.holdout_every) == (self.holdout_every - 1)
        keep = x[~hold].float()
        st.xtx += keep.t() @ keep
        if st.heldout_rows < self.holdout_cap and bool(hold.any()):
            h = x[hold].float()[: self.holdout_cap - st.heldout_rows]
            st.heldout.append(h.cpu())
            st.heldout_rows += h.shape[0]
        st.rows += n
        st.used += int(keep.shape[0])

    # ------------------------------------------------------------ results
    def hessians(self) -> dict[str, torch.Tensor]:
        """``{checkpoint linear name: H = 2 X^T X / n}`` (fp64, CPU)."""
        out: dict[str, torch.Tensor] = {}
        for fused, st in self.stats.items():
            if st.used == 0:
                continue
            H = (st.xtx.double() * (2.0 / st.used)).cpu()
            for name in checkpoint_names(fused):
                if self.select is None or self.select.search(name):
                    out[name] = H
        return out

    def heldout_inputs(self, name: str) -> torch.Tensor | None:
        """Held-out rows of the input of checkpoint linear ``name`` (CPU fp32)."""
        for fused, st in self.stats.items():
            if name in checkpoint_names(fused) and st.heldout:
                return torch.cat(st.heldout)
        return None

    def heldout_error(self, name: str, w_kn: torch.Tensor, q_kn: torch.Tensor) -> float:
        """Mean squared output error ``|X (W - Q)|^2 / rows`` of a quantized
        ``[K, N]`` weight on the held-out rows of its input."""
        x = self.heldout_inputs(name)
        if x is None:
            raise KeyError("no held-out rows for %s" % name)
        d = x.double() @ (w_kn.double() - q_kn.double())
        return float((d * d).sum() / x.shape[0])

    def save(self, path: str) -> str:
        """Write :meth:`hessians` with ``torch.save`` atomically (a ``.partial``
        file renamed into place), so a reader never sees a torn file."""
        tmp = path + ".partial"
        torch.save(self.hessians(), tmp)
        os.replace(tmp, path)
        return path


def calibrate_engine(engine, prompts: list[list[int]], select: str | None = None, holdout_every: int = 64,
                     rank: int = 0) -> Calibrator:
    """Run ``prompts`` through ``engine`` (prefill plus one sampled token each)
    with the calibrator attached to its model; every TP rank must call this
    with the same prompts."""
    from ..runtime.scheduler import SamplingParams
    calib = Calibrator(engine.model, select=select, holdout_every=holdout_every)
    with calib:
        engine.generate(prompts, SamplingParams(max_tokens=1, ignore_eos=True))
    return calib


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="k8v4-calibrate")
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--checkpoint", help="load weights from this GPTQ checkpoint instead of random init")
    ap.add_argument("--prompts", type=int, default=8, help="number of synthetic calibration prompts")
    ap.add_argument("--len", type=int, default=512, help="tokens per synthetic prompt")
    ap.add_argument("--token-file", help="JSON list of token-id lists to use as prompts")
    ap.add_argument("--select", help="regex on checkpoint linear names (default: every linear)")
    ap.add_argument("--holdout-every", type=int, default=64)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out", required=True)
    args = ap.parse_args(argv)

    from ..models.config import PRESETS
    from ..parallel.comm import TPComm, init_from_env
    from ..runtime.engine import EngineConfig, LLMEngine
    rank, world, local = init_from_env()
    comm = TPComm() if world > 1 else None
    if args.token_file:
        with open(args.token_file) as f:
            prompts = [list(map(int, p)) for p in json.load(f)]
    else:
        gen = torch.Generator().manual_seed(args.seed)
        vocab = PRESETS[args.preset].vocab
        prompts = [torch.randint(0, vocab, (args.len,), generator=gen).tolist() for _ in range(args.prompts)]
    longest = max(len(p) for p in prompts)
    cfg = EngineConfig(model=args.preset, tensor_parallel_size=world, max_model_len=longest + 16,
                       max_num_seqs=1, cuda_graphs=False, enable_prefix_caching=False,
                       num_kv_blocks=(longest + 16) // 16 + 8, device="cuda:%d" % local)
    mcfg = PRESETS[args.preset]
    if args.checkpoint:
        from ..models.checkpoint import load_checkpoint, read_model_config
        mcfg = read_model_config(args.checkpoint)
    engine = LLMEngine(cfg, mcfg, comm=comm, rank=rank)
    if args.checkpoint:
        load_checkpoint(engine.model, args.checkpoint)
    calib = calibrate_engine(engine, prompts, args.select, args.holdout_every, rank)
    if rank == 0:
        calib.save(args.out)
        print(json.dumps({"hessians": len(calib.hessians()), "out": args.out}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
