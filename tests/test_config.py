"""Config resolution (CLI > env > profile > defaults) and the launcher dry run (CPU)."""
import json
import subprocess
import sys

import pytest

from k8v4_xpu_b200.config import parse_compilation, parse_speculative, resolve


def test_defaults_match_the_reference_deployment():
    cfg = resolve([], env={})
    assert cfg.kv_cache_dtype == "int8_k_int4_v"
    assert cfg.max_num_batched_tokens == 4224
    assert cfg.max_num_seqs == 4 and cfg.enable_prefix_caching
    assert cfg.default_capture_sizes() == (1, 2, 3, 4)
    e = cfg.engine_config("cpu")
    assert e.max_num_batched_tokens == 4224 and e.capture_sizes == (1, 2, 3, 4)


def test_precedence_cli_over_env_over_profile():
    env = {"K8V4_MAX_NUM_SEQS": "3", "K8V4_PREFIX_CACHING": "0", "K8V4_TP": "4"}
    cfg = resolve(["--profile", "tp2"], env=env)
    assert (cfg.tensor_parallel_size, cfg.max_num_seqs, cfg.enable_prefix_caching) == (4, 3, False)
    cfg = resolve(["--profile", "tp2", "--max-num-seqs", "2", "-tp", "8"], env=env)
    assert (cfg.tensor_parallel_size, cfg.max_num_seqs) == (8, 2)
    cfg = resolve(["--profile", "tp1"], env={})
    assert (cfg.tensor_parallel_size, cfg.max_num_seqs, cfg.enable_prefix_caching) == (1, 1, False)


def test_speculative_and_compilation_configs():
    assert parse_speculative("mtp/6") == 6
    assert parse_speculative('{"method": "mtp", "num_speculative_tokens": 3}') == 3
    assert parse_speculative("none") == 0
    with pytest.raises(ValueError):
        parse_speculative("eagle/3")
    with pytest.raises(ValueError):
        parse_speculative("mtp/12")
    assert parse_compilation("FULL_DECODE_ONLY") == (True, ())
    assert parse_compilation('{"cudagraph_mode": "FULL_DECODE_ONLY", "cudagraph_capture_sizes": [7, 14]}') == (
        True, (7, 14))
    assert parse_compilation("NONE") == (False, ())
    cfg = resolve(["--speculative-config", "mtp/6"], env={})
    assert cfg.default_capture_sizes() == (7, 14, 21, 28)
    assert cfg.engine_config("cpu").capture_sizes == (1, 2, 3, 4)
    cfg = resolve(["--speculative-config", "mtp/6", "--compilation-config",
                   '{"cudagraph_capture_sizes": [7, 28]}'], env={})
    assert cfg.engine_config("cpu").capture_sizes == (1, 4)
    with pytest.raises(ValueError):
        resolve(["--speculative-config", "mtp/6", "--compilation-config", '{"cudagraph_capture_sizes": [8]}'],
                env={})
    assert not resolve(["--enforce-eager"], env={}).cuda_graphs


def test_validation_errors():
    with pytest.raises(ValueError):
        resolve(["--kv-cache-dtype", "fp8"], env={})
    with pytest.raises(ValueError):
        resolve(["-tp", "3"], env={})
    with pytest.raises(ValueError):
        resolve(["-tp", "8", "-cp", "2"], env={})
    with pytest.raises(ValueError):
        resolve(["--block-size", "24"], env={})


def test_dry_run_prints_every_rank():
    out = subprocess.run([sys.executable, "-m", "k8v4_xpu_b200", "serve", "--profile", "tp2", "--speculative-config",
                          "mtp/6", "--dry-run", "--port", "8123"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    plan = json.loads(out.stdout)
    assert plan["config"]["tensor_parallel_size"] == 2 and plan["config"]["capture_sizes"] == [7, 14, 21, 28]
    assert [r["role"] for r in plan["ranks"]] == ["server", "follower"]
    assert plan["ranks"][1]["env"]["RANK"] == "1" and plan["ranks"][1]["env"]["MASTER_ADDR"] == "127.0.0.1"
    assert "--dry-run" not in plan["ranks"][0]["argv"]
    assert plan["endpoint"].endswith(":8123/v1")


def test_doctor_reports_layout_library_and_devices():
    from k8v4_xpu_b200 import cli
    rep = cli.doctor()
    assert rep["layout_ok"] and rep["cache_dtype"] == "int8_k_int4_v"
    if rep["library"] is not None:  # an in-tree build must load and match its sources
        assert rep["library_loads"], rep.get("library_error")
        assert rep["library_source_hash"] == rep["tree_source_hash"]
    assert rep["ok"] == (rep["library_loads"] and (rep["gpus"] == 0 or rep["sm100"]))
    assert cli.main(["doctor"]) == (0 if rep["ok"] else 1)


def test_build_engine_picks_the_context_parallel_engine(monkeypatch):
    """--context-parallel-size > 1 builds the CP engine on this rank's CP
    group, with the TP communicator and TP rank (CP x TP); otherwise the
    plain engine."""
    import pytest
    from k8v4_xpu_b200 import cli, config
    from k8v4_xpu_b200.parallel import cp as cp_mod
    from k8v4_xpu_b200.runtime import cp_engine, engine
    made = []

    class FakeCPGroup:
        def __init__(self, group=None):
            self.group = group

    class FakeEngine:
        def __init__(self, ecfg, mcfg, *args, **kw):
            made.append((type(self).__name__, ecfg, args, kw))
            self.model = None

    class CPEngine(FakeEngine):
        pass

    class LLMEngine(FakeEngine):
        pass

    monkeypatch.setattr(cp_mod, "CPGroup", FakeCPGroup)
    monkeypatch.setattr(cp_engine, "CPEngine", CPEngine)
    monkeypatch.setattr(engine, "LLMEngine", LLMEngine)
    cfg = config.resolve(["--model", "tiny", "--context-parallel-size", "2", "--tensor-parallel-size", "2"], env={})
    cli.build_engine(cfg, comm="tp-comm", rank=1, device="cpu", cp_group="cp-group")
    name, ecfg, args, kw = made[-1]
    assert name == "CPEngine" and kw == {"rank": 1, "comm": "tp-comm"} and args[0].group == "cp-group"
    assert ecfg.context_parallel_size == 2 and ecfg.tensor_parallel_size == 2
    cfg = config.resolve(["--model", "tiny", "--tensor-parallel-size", "2"], env={})
    cli.build_engine(cfg, comm="tp-comm", rank=1, device="cpu")
    assert made[-1][0] == "LLMEngine" and made[-1][3] == {"comm": "tp-comm", "rank": 1}
    # MTP under CP resolves (the CP engine drafts through spec.mtp_cp)
    cfg = config.resolve(["--context-parallel-size", "2", "--speculative-config", "mtp/6"], env={})
    assert cfg.context_parallel_size == 2 and cfg.speculative_tokens == 6


def test_out_of_range_values_are_refused_up_front():
    import pytest
    from k8v4_xpu_b200 import config
    for argv in (["--num-kv-blocks", "-3"], ["--port", "70000"], ["--seed", "-1"], ["--layers", "0"],
                 ["--forced-accept-mean", "3.0"],
                 ["--forced-accept-mean", "0.5", "--speculative-config", "mtp/6"],
                 ["--forced-accept-mean", "8.0", "--speculative-config", "mtp/6"]):
        with pytest.raises(ValueError):
            config.resolve(argv, env={})
    assert config.resolve(["--forced-accept-mean", "3.0", "--speculative-config", "mtp/6"], env={}).forced_accept_mean == 3.0


def test_image_recipe_runs_the_build_checks_and_they_pass_here():
    """deploy/Dockerfile builds the sm_100a library and fails on a failed
    build-time check; the same checks pass on this (GPU-less) machine."""
    import pathlib
    from k8v4_xpu_b200 import cli
    root = pathlib.Path(__file__).resolve().parent.parent
    recipe = (root / "deploy" / "Dockerfile").read_text()
    runs = [ln.strip() for ln in recipe.splitlines() if ln.strip().startswith("RUN")]
    assert any("setup.py build_ext --inplace" in r for r in runs)
    assert any("k8v4_xpu_b200 doctor --build" in r for r in runs)
    assert 'ENTRYPOINT ["python", "-m", "k8v4_xpu_b200", "serve"]' in recipe
    assert "/health" in recipe
    rep = cli.build_checks()
    if rep["library"] is None:
        pytest.skip("the extension is not built in this tree")
    assert rep["build_ok"], rep
    assert cli.main(["doctor", "--build"]) == 0
