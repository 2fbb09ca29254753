"""``python -m k8v4_xpu_b200 serve ...``: launch the OpenAI-compatible server.

The launcher equivalent of the reference's ``launch.sh`` (T1) and
``tools/launch_tp1.py`` (T2):

* ``--dry-run`` prints the resolved configuration and every rank's launch
  (environment + argv) as JSON and exits (``launch.sh:196-200``);
* TP x CP > 1 starts one process per GPU (RANK / LOCAL_RANK / WORLD_SIZE,
  rendezvous on 127.0.0.1); rank 0 serves HTTP, the others mirror its steps;
* a KV-capacity error at start-up (the pool cannot hold ``--max-model-len``)
  is retried once at the fitted length; any other failure is reported and
  never retried (``launch_tp1.py:15-69``).

``python -m k8v4_xpu_b200 doctor`` prints installation checks as JSON (the
reference image's build-time checks, T3): library load, source-hash match,
page-layout asserts, devices.
"""
from __future__ import annotations

import json
import os
import signal
import socket
import subprocess
import sys

from .config import ServeConfig, resolve


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def launch_plan(cfg: ServeConfig, argv: list[str], master_port: int | None = None) -> dict:
    world = cfg.world_size
    port = master_port or 29500
    ranks = []
    for r in range(world):
        env = {"RANK": str(r), "LOCAL_RANK": str(r), "WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
               "MASTER_PORT": str(port)} if world > 1 else {}
        ranks.append({"rank": r, "role": "server" if r == 0 else "follower", "env": env,
                      "argv": [sys.executable, "-m", "k8v4_xpu_b200", "serve"] + [a for a in argv if a != "--dry-run"]})
    return {"config": cfg.to_dict(), "engine": _engine_dict(cfg), "ranks": ranks,
            "endpoint": "http://%s:%d/v1" % (cfg.host, cfg.port)}


def _engine_dict(cfg: ServeConfig) -> dict:
    import dataclasses
    d = dataclasses.asdict(cfg.engine_config())
    d["capture_sizes"] = list(d["capture_sizes"])
    return d


def build_engine(cfg: ServeConfig, comm=None, rank: int = 0, device: str = "cuda", cp_group=None):
    """Engine with the capacity-fit retry: only a CapacityError is retried.

    ``rank`` is the TP rank and ``comm`` the TP group's communicator; with
    ``--context-parallel-size`` > 1, ``cp_group`` is this rank's CP group
    (``parallel.groups``) and the engine is the context-parallel one."""
    from .models.config import PRESETS
    from .runtime.block_manager import CapacityError
    from .runtime.engine import LLMEngine
    mcfg = PRESETS.get(cfg.model)
    if mcfg is None:
        from .models.checkpoint import read_model_config
        mcfg = read_model_config(cfg.checkpoint or cfg.model)

    def make(ecfg):
        if cfg.context_parallel_size > 1:
            from .parallel.cp import CPGroup
            from .runtime.cp_engine import CPEngine
            return CPEngine(ecfg, mcfg, CPGroup(cp_group), rank=rank, comm=comm)
        return LLMEngine(ecfg, mcfg, comm=comm, rank=rank)

    try:
        eng = make(cfg.engine_config(device))
    except CapacityError as e:
        if not cfg.fit_capacity or not e.fit_tokens:
            raise
        fit = (e.fit_tokens // cfg.block_size) * cfg.block_size
        print("[k8v4] %s; retrying at max_model_len=%d" % (e, fit), file=sys.stderr, flush=True)
        cfg.max_model_len = fit
        eng = make(cfg.engine_config(device))
    if cfg.checkpoint:
        from .models.checkpoint import load_checkpoint
        load_checkpoint(eng.model, cfg.checkpoint)
    return eng


def gpu_checks(cfg: ServeConfig, local: int, nvml=None):
    """Start-up GPU checks of one rank (the reference launcher's fault-log
    warning and card settings, ``launch.sh:201-213``): local rank 0 prints
    NVML's warnings about every GPU (read only), and each rank applies the
    opt-in power limit / clock range to its own GPU. Returns (nvml, what was
    changed) when something was set, for ``gpu_setup.restore`` at exit."""
    from .tools import gpu_setup
    nvml = nvml or gpu_setup.load_nvml()
    if nvml is None:
        return None
    if local == 0:
        for w in gpu_setup.preflight(nvml):
            print("WARN: " + w, file=sys.stderr, flush=True)
    done = gpu_setup.apply_settings(nvml, [local], cfg.gpu_power_limit,
                                    gpu_setup.parse_clock_range(cfg.gpu_clock_range))
    return (nvml, done) if done else None


def run_rank(cfg: ServeConfig) -> int:
    import torch
    import torch.distributed as dist

    from .api.driver import EngineDriver, TPControl, follower_loop
    from .parallel import groups
    from .parallel.comm import TPComm, init_from_env
    rank, world, local = init_from_env(timeout_s=600)
    device = "cuda:%d" % local
    gpu_settings = gpu_checks(cfg, local)
    pg = groups.build(cfg.tensor_parallel_size, cfg.context_parallel_size)
    comm = TPComm(pg.tp_group) if pg.tp > 1 else None
    control = TPControl(dist.new_group(backend="gloo")) if world > 1 else None
    eng = build_engine(cfg, comm=comm, rank=pg.tp_rank, device=device, cp_group=pg.cp_group)
    watchdog = hb = None
    if world > 1:
        from .parallel.health import Heartbeat, Watchdog
        hb = Heartbeat(dist.distributed_c10d._get_default_store(), rank, world).start()
        watchdog = Watchdog(hb, timeout=float(os.environ.get("K8V4_HEARTBEAT_TIMEOUT", "30")))
    try:
        if rank == 0:
            import uvicorn

            from .api.metrics import ServingMetrics
            from .api.server import build_app
            from .api.tokenizer import load_tokenizer
            metrics = ServingMetrics(cfg.served_model_name or cfg.model)
            driver = EngineDriver(eng, metrics=metrics, control=control, watchdog=watchdog).start()
            app = build_app(driver, load_tokenizer(cfg.tokenizer, eng.mcfg.vocab), cfg.served_model_name or cfg.model,
                            cfg.max_model_len, metrics)
            uvicorn.run(app, host=cfg.host, port=cfg.port, log_level="info")
            driver.stop()
        else:
            follower_loop(eng, control, watchdog)
    finally:
        if hb is not None:
            hb.stop()
        if eng.graphs is not None:
            eng.graphs.release()
        if eng.mtp is not None:
            eng.mtp.release()
        torch.cuda.synchronize()
        if gpu_settings:
            from .tools import gpu_setup
            gpu_setup.restore(gpu_settings[0], gpu_settings[1])
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
    return 0


def serve(argv: list[str]) -> int:
    cfg = resolve(argv)
    if cfg.dry_run:
        print(json.dumps(launch_plan(cfg, argv), indent=2))
        return 0
    if cfg.world_size == 1 or "RANK" in os.environ:
        return run_rank(cfg)
    plan = launch_plan(cfg, argv, _free_port())
    procs = []
    for r in plan["ranks"]:
        env = dict(os.environ)
        env.update(r["env"])
        procs.append(subprocess.Popen(r["argv"], env=env))

    def forward(sig, _frame):
        for p in procs:
            if p.poll() is None:
                p.send_signal(sig)
    signal.signal(signal.SIGINT, forward)
    signal.signal(signal.SIGTERM, forward)
    rc = 0
    for p in procs:
        rc = p.wait() or rc
    return rc


def doctor() -> dict:
    """Installation checks (the reference image's build-time checks,
    ``Dockerfile.unified:18-24``: library load, layout asserts). Returns a
    report; ``ok`` is False when something a GPU run needs is missing."""
    import torch

    from . import ops
    from .buildhash import source_hash
    from .kv.layout import CACHE_DTYPE, b200_layout
    rep: dict = {"torch": torch.__version__, "cuda_build": torch.version.cuda, "cache_dtype": CACHE_DTYPE}
    lay = b200_layout(4, 6)
    # the b200 page: 16 tokens x (128 int8 K + 64 packed V + scales) per head
    rep["page_bytes_4kv"] = lay.page_bytes
    rep["layout_ok"] = lay.page_bytes == 16 * 4 * 202 and lay.page == 16 and lay.head_dim == 128
    rep["library"] = ops._library_file()
    rep["library_loads"] = ops.load()
    if not rep["library_loads"]:
        rep["library_error"] = ops._ERROR
    else:
        rep["library_source_hash"] = str(torch.ops.k8v4.source_hash())
    csrc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc")
    if os.path.isdir(csrc):
        rep["tree_source_hash"] = source_hash(csrc)
    rep["gpus"] = torch.cuda.device_count() if torch.cuda.is_available() else 0
    devs = []
    for i in range(rep["gpus"]):
        p = torch.cuda.get_device_properties(i)
        devs.append({"name": p.name, "sm": "%d.%d" % (p.major, p.minor), "sms": p.multi_processor_count,
                     "mem_gib": round(p.total_memory / 2 ** 30, 1)})
    rep["devices"] = devs
    rep["sm100"] = bool(devs) and all(d["sm"] == "10.0" for d in devs)
    if torch.distributed.is_available() and torch.distributed.is_nccl_available():
        rep["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version()) if rep["gpus"] else "available"
    from .tools import gpu_setup
    nvml = gpu_setup.load_nvml() if rep["gpus"] else None
    rep["gpu_warnings"] = gpu_setup.preflight(nvml) if nvml is not None else []  # read-only NVML queries
    rep["ok"] = bool(rep["layout_ok"] and rep["library_loads"] and (rep["gpus"] == 0 or rep["sm100"]))
    return rep


def build_checks() -> dict:
    """The deployment image's build-time checks, which need no GPU (behaviour
    of the reference's ``Dockerfile.unified:18-24``: byte-compile, patcher
    run, library load, layout asserts). Every module of the package
    byte-compiles; the in-tree library loads and was built from the ``csrc/``
    tree beside it; its op registry is complete; the cache dtype and the vLLM
    plugin register; the page layouts tile their pages. ``ok`` is the
    conjunction."""
    import compileall

    import torch

    from . import registry
    from .kv.layout import CACHE_DTYPE, b200_layout, ref_layout
    rep = doctor()
    pkg = os.path.dirname(os.path.abspath(__file__))
    rep["byte_compiled"] = bool(compileall.compile_dir(pkg, quiet=1, force=True))
    rep["hash_matches"] = bool(rep.get("library_loads")) and rep.get("library_source_hash") == rep.get(
        "tree_source_hash", rep.get("library_source_hash"))
    want_ops = ("kv_store", "rope_store", "decode_attn", "prefill_attn", "wq_gemm", "wq_gemm_allreduce", "rmsnorm",
                "silu_mul", "quant_rows", "embed_int8", "argmax", "gather_dequant", "prefill_attn_cp",
                "decode_combine_ranks", "decode_attn_push")
    rep["missing_ops"] = [o for o in want_ops if not (rep.get("library_loads") and hasattr(torch.ops.k8v4, o))]
    rep["registry"] = registry.kv_cache_torch_dtype(CACHE_DTYPE) == torch.uint8
    rep["pages_tile"] = all(lay.regions_fill_page() for lay in
                            (b200_layout(4), b200_layout(2), b200_layout(1, 3), ref_layout(2), ref_layout(4)))
    rep["build_ok"] = bool(rep["byte_compiled"] and rep["library_loads"] and rep["hash_matches"]
                           and not rep["missing_ops"] and rep["registry"] and rep["pages_tile"]
                           and rep["layout_ok"])
    return rep


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print("usage: python -m k8v4_xpu_b200 serve [options]   (serve --help for options)\n"
              "       python -m k8v4_xpu_b200 doctor            (installation checks, JSON)\n"
              "       python -m k8v4_xpu_b200 doctor --build    (image build-time checks, no GPU needed)")
        return 0
    cmd, rest = argv[0], argv[1:]
    if cmd == "serve":
        return serve(rest)
    if cmd == "doctor":
        if "--build" in rest:
            rep = build_checks()
            print(json.dumps(rep, indent=2))
            return 0 if rep["build_ok"] else 1
        rep = doctor()
        print(json.dumps(rep, indent=2))
        return 0 if rep["ok"] else 1
    print("unknown command %r" % cmd, file=sys.stderr)
    return 2
