"""Generates the golden vectors of the W4A16 path by running the reference itself.

Run in a container that has the reference checked out (read-only) at
REFERENCE_SRC (default /root/reference/src) and torch on the CPU:

    python tests/golden/make_golden.py

It imports the reference's `roofline.kernels.pack_weights` (which runs as
torch CPU ops) and `reference_gemv`, feeds them seeded inputs drawn by the
oracle's generators (numpy PCG64, reproducible on any machine), and writes:

  tests/golden/golden_small.npz   raw inputs/outputs of small cases
  tests/golden/golden_hashes.json SHA-256 of packed/scales for every workload
                                  shape (column chunks for the largest)

The reference's dequantize_v1 / gemv_v2 / gemv_v3 are Triton GPU kernels and
cannot run on the CPU; the GEMV goldens apply the reference's own
reference_gemv (kernels.py:271-273) to the v1 dequantisation restated in
oracle/w4_oracle.py, exactly the "want" of tests/test_kernels.py:61-63.
Nothing at test time reads the reference: only these committed files.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
REFERENCE_SRC = os.environ.get("REFERENCE_SRC", "/root/reference/src")
sys.path.insert(0, REFERENCE_SRC)

from roofline.kernels import pack_weights as ref_pack  # noqa: E402  (the reference)
from roofline.kernels import reference_gemv as ref_gemv  # noqa: E402

from oracle import w4_oracle as o  # noqa: E402

# (name, K, N, generator) of the workload shapes. "normal" = N(0, 0.02),
# "absmax" = the reference tests' randn / column-absmax.
HASH_CASES = [
    ("q_proj", 1536, 1536, "normal"),
    ("mlp_gate_up", 1536, 8960, "normal"),
    ("mlp_down", 8960, 1536, "normal"),
    ("kv_proj", 1536, 256, "normal"),
    ("small_attn", 1024, 1024, "normal"),
    ("small_mlp", 1024, 2816, "normal"),
    ("gemm_4096x14336", 4096, 14336, "normal"),
    ("ci_256x512", 256, 512, "normal"),
    ("absmax_q_proj", 1536, 1536, "absmax"),
    ("absmax_mlp_gate", 1536, 8960, "absmax"),
    ("absmax_mlp_down", 8960, 1536, "absmax"),
    ("absmax_1024x2816", 1024, 2816, "absmax"),
]
CHUNKED_CASES = [  # packed by column chunks of CHUNK_N (packing is column-independent)
    ("large_8192x28672", 8192, 28672, "normal"),
    ("large_28672x8192", 28672, 8192, "normal"),
    ("vocab_8192x128256", 8192, 128256, "normal"),
]
CHUNK_N = 4096
SEED = 0


def weights(K, N, kind, seed=SEED):
    return o.normal_weights(K, N, seed) if kind == "normal" else o.absmax_weights(K, N, seed)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_pack_np(w: np.ndarray):
    p, s = ref_pack(torch.from_numpy(w))
    return p.numpy(), s.numpy()


def edge_case_weights() -> np.ndarray:
    """K=256 x N=16 fp16 with the packer's corner cases, one per column."""
    K, N = 256, 16
    w = np.zeros((K, N), dtype=np.float32)
    rng = np.random.default_rng(99)
    # col 0: exact .5 ties of w/s (amax = 7 -> s = 1): round half to even
    w[:, 0] = np.tile(np.array([7, -7, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, 6.5],
                               dtype=np.float32), 22)[:K]
    # col 1: all zero (scale underflows to 0, w/s = 0/0 = NaN) in both groups
    # col 2: one tiny non-zero per group (scale underflows, w/s = +-inf)
    w[5, 2], w[130, 2] = 1e-7, -1e-7
    # col 3: fp16 subnormals
    w[:, 3] = rng.standard_normal(K) * 1e-6
    # col 4: fp16 extremes
    w[:, 4] = rng.uniform(-65504, 65504, K)
    w[0, 4] = 65504
    # col 5: single large outlier per group
    w[:, 5] = rng.standard_normal(K) * 0.01
    w[17, 5], w[200, 5] = 3.0, -5.0
    # col 6: negative zeros and zeros mixed with values
    w[:, 6] = -0.0
    w[::3, 6] = rng.standard_normal(len(w[::3, 6])) * 0.1
    # col 7: all equal positive values; col 8: all equal negative values
    w[:, 7] = 0.25
    w[:, 8] = -0.125
    # col 9: +inf in group 0 (s = inf: finite/inf = 0, inf/inf = NaN)
    w[:, 9] = rng.standard_normal(K)
    w[3, 9] = np.inf
    # col 10: values on the clamp edges (w/s just beyond +-7.5)
    w[:, 10] = np.tile(np.array([7.0, -7.0, -7.4, 7.49, -7.5], dtype=np.float32), 52)[:K]
    # cols 11..15: N(0, 0.02) like the workload
    w[:, 11:] = rng.standard_normal((K, 5)) * 0.02
    return w.astype(np.float16)


def main() -> None:
    out: dict = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                 "seed": SEED, "chunk_n": CHUNK_N, "cases": {}, "chunked": {}}
    small: dict[str, np.ndarray] = {}

    for name, K, N, kind in HASH_CASES:
        w = weights(K, N, kind)
        p, s = ref_pack_np(w)
        out["cases"][name] = {"K": K, "N": N, "kind": kind, "packed_sha256": sha(p),
                              "scales_sha256": sha(s)}
        print(name, K, N, flush=True)

    for name, K, N, kind in CHUNKED_CASES:
        w = weights(K, N, kind)
        ph, sh = [], []
        for c0 in range(0, N, CHUNK_N):
            p, s = ref_pack_np(np.ascontiguousarray(w[:, c0:c0 + CHUNK_N]))
            ph.append(sha(p))
            sh.append(sha(s))
        out["chunked"][name] = {"K": K, "N": N, "kind": kind, "packed_sha256": ph,
                                "scales_sha256": sh}
        print(name, K, N, flush=True)
        del w

    # Small raw cases with GEMV goldens (fp16 and bf16 activations, M = 1 and 4).
    for name, K, N, kind in [("normal_256x512", 256, 512, "normal"),
                             ("absmax_128x64", 128, 64, "absmax"),
                             ("normal_1024x96", 1024, 96, "normal")]:
        w = weights(K, N, kind)
        p, s = ref_pack_np(w)
        small[f"{name}/w"] = w
        small[f"{name}/packed"] = p
        small[f"{name}/scales"] = s
        wdq = torch.from_numpy(o.dequantize_fp16(p, s))
        for M in (1, 4):
            x = o.activations(M, K, seed=M)
            small[f"{name}/x_f16_m{M}"] = x
            small[f"{name}/y_f16_m{M}"] = ref_gemv(torch.from_numpy(x), wdq).numpy()
            xb = o.activations(M, K, seed=M, bf16=True)
            small[f"{name}/x_bf16_m{M}"] = xb
            xt = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
            small[f"{name}/y_bf16_m{M}"] = (xt.float() @ wdq.float()).numpy()

    w = edge_case_weights()
    p, s = ref_pack_np(w)
    small["edge/w"] = w
    small["edge/packed"] = p
    small["edge/scales"] = s

    np.savez_compressed(HERE / "golden_small.npz", **small)
    (HERE / "golden_hashes.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", HERE / "golden_small.npz", HERE / "golden_hashes.json")


if __name__ == "__main__":
    main()
