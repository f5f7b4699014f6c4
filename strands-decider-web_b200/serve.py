"""The 24-layer linear stack of BASELINE configs 4 and 5, and its two multi-GPU modes.

The stack is the int4 part of the engine's per-layer step list (``plan()``, web/public/engine/
engine.js:253-282): every layer runs its fused input projection (linear-attention qkv|z|a|b, K=2048,
N=8224, or attention q|k|v, N=3072), the out projection (2048 -> 2048), the MLP gate|up (2048 ->
12288), SiLU*mul (wgsl.js:81-90) and down (6144 -> 2048); layers follow the 3:1 pattern of the
hybrid decoder (three linear-attention layers, then one attention layer). The residual stream and
its norms follow the engine exactly (ADD_NORM, wgsl.js:55-78, engine.js:255, 277, 284): ``x`` is
fp32; before the input projection ``x += y`` (the previous layer's down output; not at layer 0) and
``h = rmsnorm(x)``; before gate|up ``x += y`` (the out projection's output) and ``h = rmsnorm(x)``;
after the last layer ``x += y`` and the final norm gives the output. The mixers between the input
and out projections (conv, recurrence, attention) are outside this path; the out projection reads
columns [0, 2048) of the input projection's output in their place. Norm weights are ones.

Multi-GPU (one process per GPU, ``torch.distributed``):

* data-parallel serving (config 5): independent requests are assigned to ranks by longest-
  processing-time order (:func:`lpt_shard`); every rank holds all weights; there is no collective.
* column-sharded prefill (config 4): each rank holds an N/g slice of every projection's output
  rows (gate and up slices kept together so SiLU*mul stays local) and the slices are all-gathered
  after every projection: by NCCL (:func:`stack_forward` on a sharded :class:`CudaStack`), or fused
  into the producing kernels, which store into every rank's buffer over NVLink
  (:class:`FusedColshardStack`).

The sharding logic takes its matmul / SiLU*mul / all-gather as callables, so the same code runs on
the CUDA kernels with NCCL and on CPU ranks with gloo in the tests.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np

HIDDEN = 2048
INTER = 6144
N_LINEAR_IN = 8224   # qkv | z | a | b of a linear-attention layer (export_engine.py:52-53, unpadded)
N_ATTN_IN = 3072     # q | k | v of an attention layer: 16 q + 4 kv heads x 128 (export_engine.py:61-62)
N_LAYERS = 24


def layer_kinds(n_layers: int = N_LAYERS):
    """``linear`` x3 then ``attn``, repeated (the 18 + 6 hybrid pattern)."""
    return ["attn" if (i % 4) == 3 else "linear" for i in range(n_layers)]


def projection_shapes(kind: str):
    """(name, K, N) of the four int4 projections of one layer, in call order."""
    n_in = N_LINEAR_IN if kind == "linear" else N_ATTN_IN
    return [("in_proj", HIDDEN, n_in), ("out_proj", HIDDEN, HIDDEN), ("gate_up", HIDDEN, 2 * INTER), ("down", INTER, HIDDEN)]


def stack_flops_per_token(n_layers: int = N_LAYERS) -> float:
    """2 * (weight parameters of the stack): multiply-adds per token of the linear path."""
    return 2.0 * sum(K * N for kind in layer_kinds(n_layers) for _, K, N in projection_shapes(kind))


# --------------------------------------------------------------------------------------------------
# request sharding for data-parallel serving
# --------------------------------------------------------------------------------------------------
def lpt_shard(lengths, world: int):
    """Longest-processing-time assignment of requests to ``world`` ranks by token count.

    Requests are taken longest first (ties by index) and each goes to the currently least-loaded
    rank (ties by rank). Returns a list of index lists, one per rank, each in ascending order.
    Deterministic; the max load is within one request of the mean (LPT's 4/3 bound in general)."""
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    out = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(v) for v in out]


def request_lengths(n: int = 4096, lo: int = 64, hi: int = 2048, seed: int = 0):
    """Config-5 request lengths: uniform integers in [lo, hi], numpy default_rng(seed)."""
    return np.random.default_rng(seed).integers(lo, hi + 1, n)


def pack_chunks(lengths, max_tokens: int):
    """Group a rank's requests into chunks of at most ``max_tokens`` tokens (a request is never
    split: the stack is row-independent, so packing only changes M). Returns lists of indices."""
    chunks, cur, cur_tok = [], [], 0
    for i, n in enumerate(lengths):
        if cur and cur_tok + n > max_tokens:
            chunks.append(cur)
            cur, cur_tok = [], 0
        cur.append(i)
        cur_tok += int(n)
    if cur:
        chunks.append(cur)
    return chunks


# --------------------------------------------------------------------------------------------------
# column sharding
# --------------------------------------------------------------------------------------------------
def shard_rows(name: str, N: int, rank: int, world: int):
    """Row indices (output columns) of projection ``name`` held by ``rank``.

    Every projection is split into ``world`` equal contiguous slices, except gate|up, whose rank
    slice is (gate slice) followed by (the matching up slice), so SiLU*mul runs on local data."""
    if name == "gate_up":
        inter = N // 2
        assert inter % world == 0
        s = inter // world
        return np.concatenate([np.arange(rank * s, (rank + 1) * s), inter + np.arange(rank * s, (rank + 1) * s)])
    assert N % world == 0, f"{name}: N={N} not divisible by {world}"
    s = N // world
    return np.arange(rank * s, (rank + 1) * s)


def gathered_to_rows(g, M: int, world: int, ns: int):
    """All-gather output [world][M][ns] (rank-major) -> [M][world * ns]."""
    return g.reshape(world, M, ns).transpose(1, 0, 2).reshape(M, world * ns) if isinstance(g, np.ndarray) else \
        g.view(world, M, ns).permute(1, 0, 2).reshape(M, world * ns)


@dataclass
class Ops:
    """The operators a stack forward needs; CUDA kernels + NCCL, or the CPU oracle + gloo."""
    matmul: object      # (x [M,K] f16, weight handle) -> y [M,N] f16
    silu_mul: object    # (big [M, 2I] f16, I) -> mid [M, I] f16; None: the gate_up matmul already wrote mid
    all_gather: object  # (local [M, ns]) -> [world][M][ns] stacked (None when world == 1)
    add_norm: object    # (x f32 [M, D], y f16 or None) -> (x + y f32, rmsnorm(x + y) f16)
    cols: object        # (x, c0, c1) -> contiguous x[:, c0:c1]
    to_f32: object      # x f16 -> fp32 residual stream (a new tensor)
    # (act f16, weight, x f32) -> (x + act @ W^T, rmsnorm of it f16) as one call, the add in the
    # projection's epilogue; None: matmul, then add_norm. Used on one GPU (no gather in between).
    matmul_add_norm: object = None


def stack_forward(x, layers, ops: Ops, world: int = 1, timers=None):
    """Run the linear stack on embeddings ``x`` [M, 2048] (fp16); returns the final-normed hidden
    states (fp16).

    ``layers`` is a list of dicts name -> weight handle (the rank's shard when ``world`` > 1); the
    norms are replicated on every rank. ``timers``, if given, is called as timers("gather", fn)
    around every all-gather."""
    M = x.shape[0]

    def gather(local):
        if world == 1:
            return local
        ns = local.shape[1]
        g = timers("gather", lambda: ops.all_gather(local)) if timers else ops.all_gather(local)
        return gathered_to_rows(g, M, world, ns)

    def proj_norm(act, wt, x):
        """A projection whose output is added to the residual stream and normalised (ADD_NORM)."""
        if ops.matmul_add_norm is not None and world == 1:
            return ops.matmul_add_norm(act, wt, x)
        return ops.add_norm(x, gather(ops.matmul(act, wt)))

    x = ops.to_f32(x)
    x, h = ops.add_norm(x, None)                                    # layer 0's in_norm (engine.js:255)
    for w in layers:
        a = gather(ops.matmul(h, w["in_proj"]))
        x, h = proj_norm(ops.cols(a, 0, HIDDEN), w["out_proj"], x)  # out_proj + post_norm (engine.js:277)
        gu = ops.matmul(h, w["gate_up"])
        mid = gather(gu if ops.silu_mul is None else ops.silu_mul(gu, gu.shape[1] // 2))
        x, h = proj_norm(mid, w["down"], x)                         # down + the next in_norm / final norm
    return h                                                        # (engine.js:255, 284)


# --------------------------------------------------------------------------------------------------
# synthetic weights (nibbles uniform, fp16 scales |N(0, 0.02)| / 7)
# --------------------------------------------------------------------------------------------------
def synthetic_projection(seed: int, K: int, N: int):
    """MatMulNBits bytes of one projection (numpy), from its own seed."""
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, size=(N, K // 32, 32), dtype=np.uint8)
    packed = (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)
    scales = (np.abs(rng.standard_normal((N, K // 32)) * 0.02) / 7.0).astype(np.float16)
    return packed, scales


def synthetic_projection_torch(seed: int, K: int, N: int, device):
    """Same distribution, generated on the GPU (fast for the 758 MB stack); returns torch tensors."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    packed = torch.randint(0, 256, (N, K // 32, 16), dtype=torch.uint8, device=device, generator=g)
    scales = (torch.randn((N, K // 32), device=device, generator=g).abs() * (0.02 / 7.0)).to(torch.float16)
    return packed, scales


def projection_seed(layer: int, name: str) -> int:
    return 1000 * (layer + 1) + ["in_proj", "out_proj", "gate_up", "down"].index(name)


class CudaStack:
    """The stack's weights uploaded through the C ABI, optionally as this rank's column shard.
    With ``fuse_silu`` (default) every gate|up projection is uploaded as a fused weight whose matmul
    writes SiLU*mul directly (``s4_weight_upload_glu``), so no separate SiLU*mul pass runs. With
    ``fuse_norm`` out_proj and down add their output to the residual stream in the GEMM epilogue and
    normalise in one row pass (``s4_matmul_add_rmsnorm``) on one GPU. It is off by default: at the
    stack's 2048-token shapes every CTA holds one tile, so the epilogue's fp32 residual traffic
    cannot hide behind a next tile's MMAs, and the one-call form measured 3-5 us slower per
    projection than the GEMM followed by the separate ADD_NORM kernel."""

    def __init__(self, ctx, n_layers: int = N_LAYERS, rank: int = 0, world: int = 1, device=None, host_gen=False,
                 fuse_silu: bool = True, fuse_norm: bool = False):
        import torch
        self.ctx, self.rank, self.world = ctx, rank, world
        self.fuse_silu = fuse_silu
        self.fuse_norm = fuse_norm
        self.device = device or torch.device("cuda", ctx.device)
        self.layers = []
        self.n_layers = n_layers
        for li, kind in enumerate(layer_kinds(n_layers)):
            ws = {}
            for name, K, N in projection_shapes(kind):
                seed = projection_seed(li, name)
                if host_gen:
                    packed, scales = synthetic_projection(seed, K, N)
                    packed, scales = torch.from_numpy(packed).to(self.device), torch.from_numpy(scales).to(self.device)
                else:
                    packed, scales = synthetic_projection_torch(seed, K, N, self.device)
                if world > 1:
                    rows = torch.from_numpy(shard_rows(name, N, rank, world)).to(self.device)
                    packed, scales = packed.index_select(0, rows).contiguous(), scales.index_select(0, rows).contiguous()
                if name == "gate_up" and fuse_silu:  # rows: the rank's gate slice, then its up slice
                    ws[name] = ctx.upload_glu(packed, scales, packed.shape[0] // 2, K)
                else:
                    ws[name] = ctx.upload(packed, scales, packed.shape[0], K)
                del packed, scales
            self.layers.append(ws)

    def ops(self, group=None):
        import torch
        import torch.distributed as dist
        ctx, world = self.ctx, self.world

        def all_gather(local):
            out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
            dist.all_gather_into_tensor(out, local.contiguous(), group=group)
            return out

        def add_norm(x, y):
            return x, ctx.add_rmsnorm(x, y)

        def matmul_add_norm(act, w, x):
            return x, ctx.matmul_add_rmsnorm(act, w, x)

        return Ops(matmul=lambda x, w: ctx.matmul(x, w),
                   silu_mul=None if self.fuse_silu else (lambda big, I: ctx.silu_mul(big, I)),
                   all_gather=all_gather,
                   add_norm=add_norm,
                   cols=lambda x, c0, c1: x[:, c0:c1].contiguous(),
                   to_f32=lambda x: x.float(),
                   matmul_add_norm=matmul_add_norm if self.fuse_norm else None)

    def forward(self, x, group=None, timers=None):
        return stack_forward(x, self.layers, self.ops(group), self.world, timers)


def _raw_tensor(ptr: int, shape, device):
    """A torch fp16 view of device memory owned elsewhere (a library buffer or a peer mapping)."""
    import torch

    class _Holder:
        pass

    h = _Holder()
    h.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f2", "data": (int(ptr), False), "version": 3,
                                  "strides": None}
    return torch.as_tensor(h, device=device)


class FusedColshardStack:
    """Column-sharded stack whose all-gathers are fused into the producing kernels.

    Every rank allocates its gathered activation buffers (one cudaMalloc each), exports them with
    CUDA IPC and maps the peers' buffers, so each GEMM epilogue (and the SiLU*mul kernel) stores
    its column slice into all ranks' buffers over NVLink while it computes. A bounded flag barrier
    between projections orders the writes before the next projection reads them."""

    def __init__(self, ctx, group, rank: int, world: int, max_tokens: int = 2048, n_layers: int = N_LAYERS,
                 fuse_silu: bool = True, split_barrier: bool = True):
        import torch
        import torch.distributed as dist
        self.ctx, self.group, self.rank, self.world = ctx, group, rank, world
        self.split_barrier = split_barrier
        self.device = torch.device("cuda", ctx.device)
        # its forward runs the norms itself (replicated, after each gather)
        self.stack = CudaStack(ctx, n_layers, rank, world, self.device, fuse_silu=fuse_silu, fuse_norm=False)
        self.max_tokens = max_tokens
        self.widths = {"a": N_LINEAR_IN, "b": HIDDEN, "mid": INTER, "d": HIDDEN}
        sizes = {k: max_tokens * w * 2 for k, w in self.widths.items()}
        sizes["flags"] = 64
        self.local = {k: ctx.buffer_alloc(v) for k, v in sizes.items()}
        every = [None] * world
        if world > 1:
            handles = {k: ctx.ipc_handle(p) for k, p in self.local.items()}
            dist.all_gather_object(every, handles, group=group)
        self.ptrs = {k: [self.local[k] if q == rank else ctx.ipc_open(every[q][k]) for q in range(world)]
                     for k in sizes}
        self.gu = torch.empty((max_tokens, 2 * INTER // world), dtype=torch.float16, device=self.device)
        self.h = torch.empty((max_tokens, HIDDEN), dtype=torch.float16, device=self.device)
        self.x = torch.empty((max_tokens, HIDDEN), dtype=torch.float32, device=self.device)
        self.flat = {k: _raw_tensor(self.local[k], (max_tokens * w,), self.device) for k, w in self.widths.items()}
        self.graph = None
        torch.cuda.synchronize(self.device)
        if world > 1:
            dist.barrier(group=group)

    def _view(self, key, M, width):
        return self.flat[key][: M * width].view(M, width)

    def barrier(self):
        """Cross-GPU flag barrier with its epoch counted on the device (graph-replayable)."""
        if self.world > 1:
            self.ctx.peer_barrier(self.ptrs["flags"], self.rank, 0)

    def forward(self, x):
        """x: [M, 2048] fp16 embeddings, the same on every rank; returns the final-normed hidden
        states [M, 2048] fp16 (a view of this object's buffer, valid until the next call). The fp32
        residual stream and the norms are replicated; the projections are sharded."""
        if self.world > 1 and self.split_barrier:
            return self._forward_split(x)
        ctx, r, g = self.ctx, self.rank, self.world
        M = x.shape[0]
        assert M <= self.max_tokens
        xs, h = self.x[:M], self.h[:M]
        xs.copy_(x)
        y = None
        for w in self.stack.layers:
            ctx.add_rmsnorm(xs, y, h=h)                                 # in_norm
            nin = w["in_proj"].N * g
            ctx.matmul_gather(h.data_ptr(), HIDDEN, M, w["in_proj"], self.ptrs["a"], nin, r * w["in_proj"].N)
            self.barrier()
            ctx.matmul_gather(self.local["a"], nin, M, w["out_proj"], self.ptrs["b"], HIDDEN, r * (HIDDEN // g))
            self.barrier()
            ctx.add_rmsnorm(xs, self._view("b", M, HIDDEN), h=h)        # post_norm
            if self.stack.fuse_silu:  # SiLU*mul in the GEMM epilogue, stored into every rank's buffer
                ctx.matmul_gather(h.data_ptr(), HIDDEN, M, w["gate_up"], self.ptrs["mid"], INTER, r * (INTER // g))
            else:
                gu = ctx.matmul(h, w["gate_up"], M, self.gu[:M])
                ctx.silu_mul_gather(gu, INTER // g, self.ptrs["mid"], INTER, r * (INTER // g))
            self.barrier()
            ctx.matmul_gather(self.local["mid"], INTER, M, w["down"], self.ptrs["d"], HIDDEN, r * (HIDDEN // g))
            self.barrier()
            y = self._view("d", M, HIDDEN)
        ctx.add_rmsnorm(xs, y, h=h)                                     # final norm
        return h

    def _forward_split(self, x):
        """The same forward with the barrier split: each gathered GEMM is followed by a signal to
        every rank, and the next consumer of gathered data (GEMM or ADD_NORM) waits for all ranks'
        signals itself, so the wait overlaps that kernel's start (its weight stream) instead of
        taking a kernel of its own. Consumers of local data (the in_proj and gate|up GEMMs read h)
        do not wait: the wait before them already covered every rank's reads of what they
        overwrite."""
        ctx, r, g = self.ctx, self.rank, self.world
        M = x.shape[0]
        assert M <= self.max_tokens
        xs, h = self.x[:M], self.h[:M]
        xs.copy_(x)
        own, flags = self.local["flags"], self.ptrs["flags"]
        wait = {"wait_flags": own, "nranks": g}
        y = None
        for w in self.stack.layers:
            if y is None:
                ctx.add_rmsnorm(xs, None, h=h)                          # in_norm of layer 0
            else:
                ctx.add_rmsnorm(xs, y, h=h, **wait)                     # in_norm (waits for down)
            nin = w["in_proj"].N * g
            ctx.matmul_gather(h.data_ptr(), HIDDEN, M, w["in_proj"], self.ptrs["a"], nin, r * w["in_proj"].N)
            ctx.peer_signal(flags, r)
            ctx.matmul_gather(self.local["a"], nin, M, w["out_proj"], self.ptrs["b"], HIDDEN, r * (HIDDEN // g),
                              **wait)
            ctx.peer_signal(flags, r)
            ctx.add_rmsnorm(xs, self._view("b", M, HIDDEN), h=h, **wait)  # post_norm
            if self.stack.fuse_silu:
                ctx.matmul_gather(h.data_ptr(), HIDDEN, M, w["gate_up"], self.ptrs["mid"], INTER, r * (INTER // g))
            else:
                gu = ctx.matmul(h, w["gate_up"], M, self.gu[:M])
                ctx.silu_mul_gather(gu, INTER // g, self.ptrs["mid"], INTER, r * (INTER // g))
            ctx.peer_signal(flags, r)
            ctx.matmul_gather(self.local["mid"], INTER, M, w["down"], self.ptrs["d"], HIDDEN, r * (HIDDEN // g),
                              **wait)
            ctx.peer_signal(flags, r)
            y = self._view("d", M, HIDDEN)
        ctx.add_rmsnorm(xs, y, h=h, **wait)                             # final norm
        return h

    def capture(self, x):
        """Record ``forward(x)`` into a CUDA graph (after at least one eager call, on every rank);
        ``replay()`` then reruns the whole stack, barriers included, on ``x``'s memory."""
        import torch
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            out = self.forward(x)
        return out

    def replay(self):
        self.graph.replay()

    def close(self):
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        self.graph = None
        self.flat = {}
        if self.world > 1:
            dist.barrier(group=self.group)
        for k, ps in self.ptrs.items():
            for q, p in enumerate(ps):
                if q != self.rank:
                    self.ctx.ipc_close(p)
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # peers unmapped before anyone frees
        for p in self.local.values():
            self.ctx.buffer_free(p)
