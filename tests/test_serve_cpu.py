"""Host-side multi-GPU logic on CPU: request sharding for data-parallel serving, and the
column-sharded stack run by two gloo ranks against the unsharded oracle stack."""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package
from oracle import s4ref


def _serve_module():
    load_package()
    return importlib.import_module("strands_decider_web_b200.serve")


@pytest.fixture(scope="module")
def serve():
    return _serve_module()


def test_layer_pattern_and_flops(serve):
    kinds = serve.layer_kinds()
    assert kinds.count("linear") == 18 and kinds.count("attn") == 6
    assert kinds[:4] == ["linear", "linear", "linear", "attn"]
    # 1.3476e9 weight parameters -> 2.695 GFLOP per token
    assert abs(serve.stack_flops_per_token() / 2 - 1.3476e9) / 1.3476e9 < 1e-3


def test_lpt_shard_assigns_everything_once_and_balances(serve):
    lengths = serve.request_lengths(4096)
    assert lengths.min() >= 64 and lengths.max() <= 2048
    for world in (1, 2, 3, 8):
        parts = serve.lpt_shard(lengths, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(lengths)))
        loads = [int(lengths[p].sum()) for p in parts]
        assert max(loads) - min(loads) <= int(lengths.max())
        assert parts == serve.lpt_shard(lengths, world)  # deterministic


def test_pack_chunks(serve):
    lengths = np.array([100, 900, 50, 1000, 2000, 10])
    chunks = serve.pack_chunks(lengths, 1024)
    assert sorted(i for c in chunks for i in c) == list(range(len(lengths)))
    for c in chunks:
        assert lengths[c].sum() <= 1024 or len(c) == 1


def test_shard_rows_partition(serve):
    for name, N in (("in_proj", 8224), ("out_proj", 2048), ("gate_up", 12288), ("down", 2048)):
        for world in (1, 2, 4, 8):
            rows = [serve.shard_rows(name, N, r, world) for r in range(world)]
            assert sorted(np.concatenate(rows).tolist()) == list(range(N))
    gu = serve.shard_rows("gate_up", 16, 1, 2)
    assert gu.tolist() == [4, 5, 6, 7, 12, 13, 14, 15]  # gate slice then the matching up slice


# ---- the column-sharded stack on two gloo ranks, checked against the unsharded stack ------------------
SMALL = dict(n_layers=2, M=8)


def _oracle_layers(serve, n_layers, rank=0, world=1):
    layers = []
    for li, kind in enumerate(serve.layer_kinds(n_layers)):
        ws = {}
        for name, K, N in serve.projection_shapes(kind):
            packed, scales = serve.synthetic_projection(serve.projection_seed(li, name), K, N)
            if world > 1:
                rows = serve.shard_rows(name, N, rank, world)
                packed, scales = packed[rows], scales[rows]
            ws[name] = (packed, scales)
        layers.append(ws)
    return layers


def _add_norm(x, y):
    xn, h = s4ref.add_rmsnorm(x.numpy(), None if y is None else y.numpy())
    return torch.from_numpy(xn), torch.from_numpy(h)


def _cpu_ops(serve, world):
    def matmul(x, w):
        y, _ = s4ref.matmul(x.numpy(), *w)
        return torch.from_numpy(y)

    def all_gather(local):
        out = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(out, local.contiguous())
        return torch.stack(out)

    return serve.Ops(matmul=matmul,
                     silu_mul=lambda big, I: torch.from_numpy(s4ref.silu_mul(big.numpy(), I)),
                     all_gather=all_gather,
                     add_norm=_add_norm,
                     cols=lambda x, c0, c1: x[:, c0:c1].contiguous(),
                     to_f32=lambda x: x.float())


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        serve = _serve_module()
        x = torch.from_numpy(s4ref.config_x(np.random.default_rng(7), SMALL["M"], serve.HIDDEN))
        layers = _oracle_layers(serve, SMALL["n_layers"], rank, world)
        y = serve.stack_forward(x, layers, _cpu_ops(serve, world), world)
        q.put((rank, y.numpy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_column_sharded_stack_matches_unsharded_on_two_gloo_ranks(serve):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # unsharded reference, one process
    x = torch.from_numpy(s4ref.config_x(np.random.default_rng(7), SMALL["M"], serve.HIDDEN))
    ref = serve.stack_forward(x, _oracle_layers(serve, SMALL["n_layers"]), _cpu_ops(serve, 1), 1).numpy()
    for r in range(world):
        # same math per output element; fp32 sums in a different grouping -> fp16-level agreement
        ok, mr, mc = s4ref.check(results[r], ref.astype(np.float32))
        assert ok, (r, mr, mc)
    np.testing.assert_array_equal(results[0], results[1])
