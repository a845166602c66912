"""Host-side logic that needs no GPU: backend routing (backends.conf,
FLAGOS_OP_* overrides -- the reference tests routing the same way, through
subprocesses with env overrides: tests/integration/ops/test_softmax_dispatch
.py:25-40), the row sharding across ranks (2 gloo ranks on CPU), and the
failure path of a missing native library."""

import os
import subprocess
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from torch_fl import sharding

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "pytorch-plugin-fl_b200")


def _py(code, env=None):
    e = os.environ.copy()
    e.update(env or {})
    e["PYTHONPATH"] = os.pathsep.join([ROOT, PKG, e.get("PYTHONPATH", "")])
    return subprocess.run([sys.executable, "-c", code], env=e, capture_output=True, text=True,
                          timeout=300)


ROUTES = "import torch_fl, json; print(json.dumps(torch_fl.routes()))"


def _routes(env=None):
    import json

    r = _py(ROUTES, env)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1]), r.stderr


def test_default_config_routes_the_op_set_to_b200():
    # every routed op of the path, the HF formula ops included, runs on the
    # b200 kernels with the shipped config; no op is configured `= cuda`
    routes, _ = _routes()
    for op in ["add.Tensor", "mul.Tensor", "_softmax", "sum.dim_IntList", "mean.dim", "amax",
               "argmax", "silu", "rsqrt", "neg", "cos", "sin", "pow.Tensor_Scalar", "cat",
               "_softmax_backward_data", "silu_backward"]:
        assert routes[op] == "b200", (op, routes[op])
    conf = os.path.join(ROOT, "pytorch-plugin-fl_b200", "torch_fl", "backends.conf")
    lines = [ln.split("#")[0].strip() for ln in open(conf)]
    assert not [ln for ln in lines if ln.replace(" ", "").endswith("=cuda")]


def test_env_override_and_custom_config(tmp_path):
    routes, err = _routes({"FLAGOS_OP__softmax": "cuda", "FLAGOS_OP_sum__dim_IntList": "cuda"})
    assert routes["_softmax"] == "cuda" and routes["sum.dim_IntList"] == "cuda"
    assert "env override: _softmax -> cuda" in err
    conf = tmp_path / "b.conf"
    conf.write_text("# all on cuda except softmax\nadd.Tensor = cuda\n_softmax=b200 # trailing\n"
                    "mul.Tensor = nonsense\n")
    routes, err = _routes({"FLAGOS_BACKEND_CONFIG": str(conf)})
    assert routes["add.Tensor"] == "cuda" and routes["_softmax"] == "b200"
    assert routes["mul.Tensor"] == "b200"           # unknown backend ignored -> default
    assert "unknown backend 'nonsense'" in err
    assert routes["amax"] == "b200"                 # unlisted op with a b200 kernel
    assert routes["cat"] == "b200"                  # every routed op has one


def test_missing_config_falls_back_to_defaults(tmp_path):
    routes, _ = _routes({"FLAGOS_BACKEND_CONFIG": str(tmp_path / "absent.conf")})
    # no config: every op with a b200 kernel (all routed ops) runs on b200
    assert routes["_softmax"] == "b200" and routes["neg"] == "b200"


def test_missing_kernel_library_fails_loudly(tmp_path):
    from torch_fl import _abi

    with pytest.raises(FileNotFoundError, match="no fallback"):
        _abi.open_library(str(tmp_path / "libfl_b200.so"))


@pytest.mark.parametrize("total,world", [(131072, 1), (131072, 2), (131072, 8), (10, 3), (0, 4)])
def test_row_range_partitions(total, world):
    seen = []
    for r in range(world):
        s, n = sharding.row_range(total, world, r)
        seen.extend(range(s, s + n))
        assert abs(n - total // world) <= 1
    assert seen == list(range(total))


def _rank_main(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, n = sharding.row_range(10, world, rank)
        pos = sharding.positions(10, world, rank)
        assert pos.tolist() == list(range(start, start + n))
        sample = torch.full((2, 3), float(rank))
        g = sharding.gather_rows(sample)
        m = sharding.max_over_ranks(1.5 * (rank + 1))
        out[rank] = (g.tolist(), m)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_and_max():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_rank_main, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        g, m = out[r]
        assert g == [[[0.0] * 3] * 2, [[1.0] * 3] * 2]
        assert m == 3.0


def test_hf_hooks_install_and_leave_cpu_tensors_alone():
    """enable_hf_fused_ops patches RMSNorm, RoPE, the MLP and the eager
    attention of a model file; on CPU tensors every hook runs the original
    HF code, so a left-padded batch gives the same logits bit for bit, and
    disable_hf_fused_ops restores the originals."""
    import torch_fl
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from transformers.models.qwen3 import modeling_qwen3 as mq

    cfg = Qwen3Config(vocab_size=128, hidden_size=64, intermediate_size=128,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=16, max_position_embeddings=64, attn_implementation="eager")
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).eval()
    ids = torch.randint(0, 128, (2, 12), generator=torch.Generator().manual_seed(5))
    am = torch.ones(2, 12, dtype=torch.long)
    am[1, :3] = 0
    with torch.no_grad():
        ref = model(ids, attention_mask=am).logits
    orig = mq.eager_attention_forward
    try:
        patched = torch_fl.enable_hf_fused_ops(models=("qwen3",))
        for site in ("Qwen3RMSNorm.forward", "Qwen3MLP.forward", "apply_rotary_pos_emb",
                     "eager_attention_forward"):
            assert any(p.endswith(site) for p in patched), (site, patched)
        assert mq.eager_attention_forward.__wrapped__ is orig
        with torch.no_grad():
            out = model(ids, attention_mask=am).logits
    finally:
        torch_fl.disable_hf_fused_ops()
    assert mq.eager_attention_forward is orig
    assert torch.equal(out, ref)

