"""Generate the golden fixtures that pin the oracle to the reference's own code.

Run where the reference source tree is available (it is read, never modified)::

    python tests/golden/make_golden.py --reference <path to strands-decider-web checkout>

What it executes from the reference, unmodified:

* ``quant`` from ``convert/export_engine.py:17-26``. The module itself cannot be imported (it opens
  a model checkpoint at import time, export_engine.py:12-15), so the ``quant`` function
  definition is extracted with ``ast`` and executed alone under torch.
* the weight-generator statements of ``convert/make_gemm.py:4-10`` and ``convert/make_chain.py:22-29``
  (the ``rng`` line and the ``q`` / ``packed`` / ``scales`` assignments of each loop body), also
  extracted with ``ast``; the ONNX half of those scripts needs ``onnx``, which is absent.

Outputs (small, committed): ``quant_cases.npz`` (inputs and the reference quantiser's outputs),
``matmul_cases.npz`` (fp16 activations, the reference-quantised weights and the fp32 result of
the fake-quant route ``torch.nn.functional.linear(x.float(), deq)``, export_engine.py:88-103),
and ``generators.json`` (sha256 of every generated weight array of the two bench recipes).
"""
from __future__ import annotations

import argparse
import ast
import hashlib
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_function(path: str, name: str, env: dict):
    tree = ast.parse(open(path).read(), filename=path)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == name)
    ns = dict(env)
    exec(compile(ast.Module(body=[fn], type_ignores=[]), path, "exec"), ns)
    return ns[name]


def _generator(path: str):
    """Return a function running the script's weight-generation statements for one shape."""
    tree = ast.parse(open(path).read(), filename=path)
    rng_stmt = next(n for n in tree.body if isinstance(n, ast.Assign)
                    and getattr(n.targets[0], "id", None) == "rng")
    loop = next(n for n in tree.body if isinstance(n, ast.For))
    keep = [s for s in loop.body if isinstance(s, ast.Assign)
            and isinstance(s.targets[0], ast.Name) and s.targets[0].id in ("blocks", "q", "packed", "scales")]
    body = ast.Module(body=keep, type_ignores=[])
    code = compile(body, path, "exec")
    rng_code = compile(ast.Module(body=[rng_stmt], type_ignores=[]), path, "exec")
    shapes_stmt = [n for n in tree.body if isinstance(n, ast.Assign) and getattr(n.targets[0], "id", None) == "shapes"]

    def make_rng():
        ns = {"np": np}
        exec(rng_code, ns)
        return ns["rng"]

    def one(rng, K, N):
        ns = {"np": np, "rng": rng, "K": K, "N": N}
        exec(code, ns)
        return ns["packed"], ns["scales"]

    shapes = None
    if shapes_stmt:
        ns = {}
        exec(compile(ast.Module(body=shapes_stmt, type_ignores=[]), path, "exec"), ns)
        shapes = ns["shapes"]
    return make_rng, one, shapes


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def quant_inputs():
    """Seeded weight matrices plus the edge cases the quantiser rule has."""
    rng = np.random.default_rng(1234)
    cases = {}
    cases["normal_64x256"] = (rng.standard_normal((64, 256)) * 0.05).astype(np.float32)
    cases["wide_16x2048"] = (rng.standard_normal((16, 2048)) * 0.02).astype(np.float32)
    e = np.zeros((8, 64), dtype=np.float32)
    e[0, :32] = 0.0                                    # all-zero block -> scale 1 (export_engine.py:22)
    e[0, 32:] = np.linspace(-1, 1, 32)
    e[1, :] = np.arange(64, dtype=np.float32) - 20.0   # positive max -> negative scale
    e[2, :] = -(np.arange(64, dtype=np.float32))       # negative max -> positive scale
    e[3, :32] = 3.0                                    # ties in |max|: first index wins
    e[3, 5] = -3.0
    e[3, 32:] = [(i % 17) * 0.5 - 4.0 for i in range(32)]   # exact half steps -> round half to even
    e[4, :] = 1e-6 * (np.arange(64) - 31)              # tiny values: fp16 subnormal scale
    e[5, :] = 6e4 * np.sin(np.arange(64))              # large values near the fp16 range
    e[6, :32] = 8.0 * np.array([(-1) ** i for i in range(32)])
    e[6, 32:] = -0.0
    e[7, :] = rng.standard_normal(64).astype(np.float32)
    cases["edges_8x64"] = e
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference source tree")
    args = ap.parse_args()
    ref = args.reference

    quant = _load_function(os.path.join(ref, "convert", "export_engine.py"), "quant", {"torch": torch, "np": np})

    # 1. reference quantiser on seeded + edge-case inputs
    qz = {}
    for name, W in quant_inputs().items():
        packed, scales, deq = quant(torch.from_numpy(W.copy()))
        qz[f"{name}/W"] = W
        qz[f"{name}/packed"] = np.asarray(packed)
        qz[f"{name}/scales"] = np.asarray(scales)
        qz[f"{name}/deq"] = deq.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "quant_cases.npz"), **qz)

    # 2. reference fake-quant matmul (fp32 nn.Linear on the dequantised weights) at small shapes
    mm = {}
    rng = np.random.default_rng(99)
    for name, (M, K, N) in {"m5_k512_n256": (5, 512, 256), "m1_k2048_n96": (1, 2048, 96),
                             "m33_k96_n48": (33, 96, 48), "m8_k6144_n16": (8, 6144, 16)}.items():
        W = (rng.standard_normal((N, K)) * 0.03).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float16)
        packed, scales, deq = quant(torch.from_numpy(W))
        y32 = torch.nn.functional.linear(torch.from_numpy(x).float(), deq).numpy()
        mm[f"{name}/x"] = x
        mm[f"{name}/packed"] = np.asarray(packed)
        mm[f"{name}/scales"] = np.asarray(scales)
        mm[f"{name}/y32"] = y32.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "matmul_cases.npz"), **mm)

    # 3. the two bench weight generators, as hashes of every generated array
    gens = {}
    make_rng, one, shapes = _generator(os.path.join(ref, "convert", "make_gemm.py"))
    r = make_rng()
    gens["make_gemm"] = []
    for K, N in shapes:
        packed, scales = one(r, K, N)
        gens["make_gemm"].append({"K": K, "N": N, "packed_sha256": sha(packed), "scales_sha256": sha(scales),
                                  "scales_head": [int(v) for v in scales.view(np.uint16).ravel()[:4]]})
    make_rng, one, _ = _generator(os.path.join(ref, "convert", "make_chain.py"))
    r = make_rng()
    gens["make_chain"] = []
    for i in range(16):
        K, N = (2048, 6144) if i % 2 == 0 else (6144, 2048)
        packed, scales = one(r, K, N)
        gens["make_chain"].append({"K": K, "N": N, "packed_sha256": sha(packed), "scales_sha256": sha(scales)})
    gens["numpy"] = np.__version__
    gens["torch"] = torch.__version__
    with open(os.path.join(HERE, "generators.json"), "w") as f:
        json.dump(gens, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
