"""Typed serving configuration: CLI flags > ``K8V4_*`` environment > profile defaults.

The flag names are the ones the reference deployment passes to ``vllm serve``
(``k8v4_v030/launch.sh:176-194``): ``--kv-cache-dtype int8_k_int4_v``,
``--tensor-parallel-size``, ``--max-num-seqs``, ``--max-num-batched-tokens``
(default 4,224), ``--max-model-len``, ``--enable-prefix-caching``,
``--speculative-config`` (``mtp/6`` or the JSON form) and
``--compilation-config`` (FULL_DECODE_ONLY with capture sizes in rows, 7*i
under MTP6, ``launch.sh:65-70``). The two launcher profiles mirror
``launch.sh:10-32``: ``tp2`` (4 sequences, prefix caching) and ``tp1`` (one
sequence, no prefix caching); ``--context-parallel-size`` adds the CP
layouts the reference never had.

``resolve(argv, env)`` returns a :class:`ServeConfig` whose ``engine`` field
is the :class:`~k8v4_xpu_b200.runtime.engine.EngineConfig` every rank builds.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
from typing import Any, Mapping, Sequence

from .kv.layout import CACHE_DTYPE
from .kv.skip_layers import parse_layers, resolve_skip_dtype

PROFILES: dict[str, dict[str, Any]] = {
    # launch.sh:10-32
    "tp2": {"tensor_parallel_size": 2, "max_num_seqs": 4, "enable_prefix_caching": True},
    "tp1": {"tensor_parallel_size": 1, "max_num_seqs": 1, "enable_prefix_caching": False},
    "tp4": {"tensor_parallel_size": 4, "max_num_seqs": 4, "enable_prefix_caching": True},
    "tp8": {"tensor_parallel_size": 8, "max_num_seqs": 4, "enable_prefix_caching": True},
    "cp8": {"tensor_parallel_size": 1, "context_parallel_size": 8, "max_num_seqs": 4,
            "enable_prefix_caching": True},
    "cp4tp2": {"tensor_parallel_size": 2, "context_parallel_size": 4, "max_num_seqs": 4,
               "enable_prefix_caching": True},
}

# field -> (env var, type)
ENV: dict[str, tuple[str, type]] = {
    "model": ("K8V4_MODEL", str),
    "tensor_parallel_size": ("K8V4_TP", int),
    "context_parallel_size": ("K8V4_CP", int),
    "max_model_len": ("K8V4_MAX_MODEL_LEN", int),
    "max_num_seqs": ("K8V4_MAX_NUM_SEQS", int),
    "max_num_batched_tokens": ("K8V4_MAX_BATCHED_TOKENS", int),
    "enable_prefix_caching": ("K8V4_PREFIX_CACHING", bool),
    "gpu_memory_utilization": ("K8V4_GPU_MEMORY_UTILIZATION", float),
    "num_kv_blocks": ("K8V4_NUM_KV_BLOCKS", int),
    "speculative_tokens": ("K8V4_SPEC_TOKENS", int),
    "forced_accept_mean": ("K8V4_FORCED_ACCEPT_MEAN", float),
    "mtp_prefill_slice": ("K8V4_MTP_PREFILL_SLICE", int),
    "cuda_graphs": ("K8V4_CUDA_GRAPHS", bool),
    "seed": ("K8V4_SEED", int),
    "host": ("K8V4_HOST", str),
    "port": ("K8V4_PORT", int),
    "served_model_name": ("K8V4_SERVED_MODEL_NAME", str),
    "checkpoint": ("K8V4_CHECKPOINT", str),
    "tokenizer": ("K8V4_TOKENIZER", str),
    "dry_run": ("K8V4_DRY_RUN", bool),
    "profile": ("K8V4_PROFILE_NAME", str),
    "gpu_power_limit": ("K8V4_GPU_POWER_LIMIT", float),
    "gpu_clock_range": ("K8V4_GPU_CLOCK_RANGE", str),
}


def _parse_bool(v: str) -> bool:
    s = str(v).strip().lower()
    if s in ("1", "true", "yes", "on"):
        return True
    if s in ("0", "false", "no", "off", ""):
        return False
    raise ValueError("not a boolean: %r" % v)


def parse_speculative(spec: str | None) -> int:
    """``mtp/6`` | ``{"method": "mtp", "num_speculative_tokens": 6}`` | ``none`` -> draft tokens."""
    if spec is None:
        return 0
    s = spec.strip()
    if s.lower() in ("", "none", "off", "0"):
        return 0
    if s.startswith("{"):
        d = json.loads(s)
        method = str(d.get("method", "mtp")).lower()
        if method not in ("mtp", "qwen3_next_mtp", "deepseek_mtp"):
            raise ValueError("only MTP speculative decoding is supported, got %r" % method)
        n = int(d.get("num_speculative_tokens", 0))
    else:
        method, _, n = s.partition("/")
        if method.lower() != "mtp" or not n:
            raise ValueError("speculative config must look like mtp/<n>, got %r" % spec)
        n = int(n)
    if not 0 <= n <= 10:
        raise ValueError("MTP draft tokens must lie in [0, 10] (verify rows = (n+1) * GQA <= 64)")
    return n


def parse_compilation(cc: str | None) -> tuple[bool, tuple[int, ...]]:
    """``--compilation-config``: ``FULL_DECODE_ONLY`` / ``NONE`` or JSON with
    ``cudagraph_mode`` and ``cudagraph_capture_sizes`` (rows). Returns
    (graphs on, capture sizes in rows)."""
    if cc is None:
        return True, ()
    s = cc.strip()
    if s.startswith("{"):
        d = json.loads(s)
        mode = str(d.get("cudagraph_mode", "FULL_DECODE_ONLY")).upper()
        sizes = tuple(int(x) for x in d.get("cudagraph_capture_sizes", ()))
    else:
        mode, sizes = s.upper(), ()
    if mode in ("NONE", "EAGER", "0"):
        return False, ()
    if mode not in ("FULL_DECODE_ONLY", "FULL", "3"):
        raise ValueError("only FULL_DECODE_ONLY CUDA graphs are supported, got %r" % mode)
    return True, sizes


@dataclasses.dataclass
class ServeConfig:
    model: str = "dense-27b"
    tensor_parallel_size: int = 1
    context_parallel_size: int = 1
    kv_cache_dtype: str = CACHE_DTYPE
    max_model_len: int = 262144
    max_num_seqs: int = 4
    max_num_batched_tokens: int = 4224
    enable_prefix_caching: bool = True
    block_size: int = 16
    gpu_memory_utilization: float = 0.90
    num_kv_blocks: int | None = None
    speculative_tokens: int = 0
    forced_accept_mean: float | None = None
    mtp_prefill_slice: int = 1024
    cuda_graphs: bool = True
    capture_sizes: tuple[int, ...] = ()
    seed: int = 0
    layers: int | None = None
    host: str = "127.0.0.1"
    port: int = 8000
    served_model_name: str | None = None
    checkpoint: str | None = None
    tokenizer: str | None = None
    dry_run: bool = False
    profile: str | None = None
    fit_capacity: bool = True
    kv_cache_dtype_skip_layers: tuple[int, ...] = ()
    kv_skip_dtype: str | None = None
    # opt-in GPU settings (off unless given; they outlast the process): tools/gpu_setup.py
    gpu_power_limit: float | None = None
    gpu_clock_range: str | None = None

    @property
    def world_size(self) -> int:
        return self.tensor_parallel_size * self.context_parallel_size

    @property
    def decode_width(self) -> int:
        return 1 + self.speculative_tokens

    def default_capture_sizes(self) -> tuple[int, ...]:
        """Capture sizes in rows: multiples of the decode width (launch.sh:65-70)."""
        return tuple(self.decode_width * i for i in range(1, self.max_num_seqs + 1))

    def engine_config(self, device: str = "cuda"):
        from .runtime.engine import EngineConfig
        w = self.decode_width
        seqs = tuple(sorted({s // w for s in (self.capture_sizes or self.default_capture_sizes())
                             if s % w == 0 and 1 <= s // w <= self.max_num_seqs}))
        return EngineConfig(
            model=self.model, tensor_parallel_size=self.tensor_parallel_size,
            context_parallel_size=self.context_parallel_size, kv_cache_dtype=self.kv_cache_dtype,
            max_model_len=self.max_model_len, max_num_seqs=self.max_num_seqs,
            max_num_batched_tokens=self.max_num_batched_tokens, enable_prefix_caching=self.enable_prefix_caching,
            block_size=self.block_size, gpu_memory_utilization=self.gpu_memory_utilization,
            num_kv_blocks=self.num_kv_blocks, speculative_tokens=self.speculative_tokens,
            cuda_graphs=self.cuda_graphs, capture_sizes=seqs, seed=self.seed, layers=self.layers,
            forced_accept_mean=self.forced_accept_mean, mtp_prefill_slice=self.mtp_prefill_slice, device=device,
            kv_cache_dtype_skip_layers=self.kv_cache_dtype_skip_layers, kv_skip_dtype=self.kv_skip_dtype)

    def validate(self) -> None:
        if self.kv_cache_dtype != CACHE_DTYPE:
            raise ValueError("--kv-cache-dtype must be %s" % CACHE_DTYPE)
        for name in ("tensor_parallel_size", "context_parallel_size", "max_num_seqs", "max_num_batched_tokens",
                     "max_model_len"):
            if getattr(self, name) < 1:
                raise ValueError("%s must be positive" % name)
        if self.tensor_parallel_size not in (1, 2, 4, 8):
            raise ValueError("--tensor-parallel-size must be 1, 2, 4 or 8")
        if self.world_size > 8:
            raise ValueError("TP x CP must fit one 8-GPU node")
        if self.block_size % 16:
            raise ValueError("--block-size must be a multiple of the 16-token page")
        if not 0.0 < self.gpu_memory_utilization <= 1.0:
            raise ValueError("--gpu-memory-utilization must lie in (0, 1]")
        if self.num_kv_blocks is not None and self.num_kv_blocks < 1:
            raise ValueError("--num-kv-blocks must be positive")
        if self.layers is not None and self.layers < 1:
            raise ValueError("--layers must be positive")
        if not 0 <= self.port <= 65535:
            raise ValueError("--port must lie in [0, 65535]")
        if self.seed < 0:
            raise ValueError("--seed must be non-negative")
        if self.gpu_power_limit is not None and self.gpu_power_limit <= 0:
            raise ValueError("--gpu-power-limit must be positive (watts)")
        if self.gpu_clock_range is not None:
            from .tools.gpu_setup import parse_clock_range
            parse_clock_range(self.gpu_clock_range)
        if self.mtp_prefill_slice < 0:
            raise ValueError("--mtp-prefill-slice must be >= 0")
        if self.forced_accept_mean is not None:
            if not self.speculative_tokens:
                raise ValueError("--forced-accept-mean needs --speculative-config")
            if not 1.0 <= self.forced_accept_mean <= self.speculative_tokens + 1:
                raise ValueError("--forced-accept-mean must lie in [1, %d]" % (self.speculative_tokens + 1))
        if self.kv_cache_dtype_skip_layers:
            if self.context_parallel_size > 1:
                raise ValueError("--kv-cache-dtype-skip-layers is not supported with --context-parallel-size")
            resolve_skip_dtype(self.kv_skip_dtype or "auto")
        w = self.decode_width
        for s in self.capture_sizes:
            if s % w:
                raise ValueError("capture size %d is not a multiple of the decode width %d" % (s, w))

    def to_dict(self) -> dict:
        d = dataclasses.asdict(self)
        d["capture_sizes"] = list(self.capture_sizes or self.default_capture_sizes())
        d["world_size"] = self.world_size
        return d


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="k8v4-serve", description="Serve a K8/V4 model (OpenAI-compatible API).")
    a = ap.add_argument
    a("--model", help="model preset (dense-27b, small, tiny) or a checkpoint directory")
    a("--profile", choices=sorted(PROFILES), help="launcher profile defaults (tp2, tp1, tp4, tp8, cp8, cp4tp2)")
    a("--tensor-parallel-size", "-tp", type=int, dest="tensor_parallel_size")
    a("--context-parallel-size", "-cp", type=int, dest="context_parallel_size")
    a("--kv-cache-dtype")
    a("--max-model-len", type=int)
    a("--max-num-seqs", type=int)
    a("--max-num-batched-tokens", type=int)
    a("--enable-prefix-caching", action="store_true", default=None)
    a("--no-enable-prefix-caching", action="store_false", dest="enable_prefix_caching")
    a("--block-size", type=int)
    a("--gpu-memory-utilization", type=float)
    a("--num-kv-blocks", type=int)
    a("--speculative-config", help="mtp/6 or JSON")
    a("--forced-accept-mean", type=float, help="benchmark mode: seeded Bernoulli acceptance with this mean length")
    a("--mtp-prefill-slice", type=int,
      help="under MTP: prefill tokens run beside each speculative decode step (0: alternate whole steps)")
    a("--compilation-config", help="FULL_DECODE_ONLY, NONE, or JSON with cudagraph_capture_sizes")
    a("--enforce-eager", action="store_true", default=None)
    a("--seed", type=int)
    a("--layers", type=int, help="debug: run only this many decoder layers")
    a("--host")
    a("--port", type=int)
    a("--served-model-name")
    a("--checkpoint", help="GPTQ + INT8 side-file checkpoint directory (default: random init)")
    a("--tokenizer", help="tokenizer directory (default: byte-level)")
    a("--dry-run", action="store_true", default=None)
    a("--no-fit-capacity", action="store_false", dest="fit_capacity", default=None)
    a("--kv-cache-dtype-skip-layers", help="comma-separated layers whose KV stays in --kv-skip-dtype "
      "(the MTP layer's index is the layer count)")
    a("--kv-skip-dtype", help="skip layers' KV dtype: auto (bf16), bfloat16, fp8, fp8_e4m3, fp8_e5m2")
    a("--gpu-power-limit", type=float, help="opt-in: set each GPU's power limit (W) at start, restored at exit")
    a("--gpu-clock-range", help="opt-in: lock each GPU's SM clocks to MIN,MAX MHz at start, unlocked at exit")
    return ap


def resolve(argv: Sequence[str] | None = None, env: Mapping[str, str] | None = None) -> ServeConfig:
    env = os.environ if env is None else env
    ns = build_parser().parse_args(list(argv) if argv is not None else None)
    cli = {k: v for k, v in vars(ns).items() if v is not None}
    values: dict[str, Any] = {}
    profile = cli.get("profile") or env.get("K8V4_PROFILE_NAME")
    if profile:
        if profile not in PROFILES:
            raise ValueError("unknown profile %r" % profile)
        values.update(PROFILES[profile])
        values["profile"] = profile
    for field, (var, typ) in ENV.items():
        if var in env and env[var] != "":
            raw = env[var]
            values[field] = _parse_bool(raw) if typ is bool else typ(raw)
    spec_cli = cli.pop("speculative_config", None)
    spec_env = env.get("K8V4_SPECULATIVE_CONFIG")
    if spec_cli is not None or spec_env:
        values["speculative_tokens"] = parse_speculative(spec_cli if spec_cli is not None else spec_env)
    cc = cli.pop("compilation_config", None) or env.get("K8V4_COMPILATION_CONFIG")
    if cc is not None:
        values["cuda_graphs"], values["capture_sizes"] = parse_compilation(cc)
    if cli.pop("enforce_eager", False):
        values["cuda_graphs"] = False
    skip = cli.pop("kv_cache_dtype_skip_layers", None) or env.get("K8V4_KV_SKIP_LAYERS")
    if skip:
        values["kv_cache_dtype_skip_layers"] = parse_layers(skip)
        # the reference deployment's VLLM_KV_SKIP_DTYPE is honoured after K8V4_KV_SKIP_DTYPE
        values["kv_skip_dtype"] = resolve_skip_dtype(cli.pop("kv_skip_dtype", None), env)
    values.update(cli)
    if values.get("served_model_name") is None:
        values["served_model_name"] = str(values.get("model", ServeConfig.model))
    cfg = ServeConfig(**{k: v for k, v in values.items() if k in {f.name for f in dataclasses.fields(ServeConfig)}})
    if isinstance(cfg.capture_sizes, list):
        cfg.capture_sizes = tuple(cfg.capture_sizes)
    cfg.validate()
    return cfg
