"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own code.

Run where the QVex reference tree is on disk ($QVEX_REFERENCE, or a directory named
``reference`` beside this repository):

    python tests/golden/make_golden.py [reference_root]

Sources of truth, all executed from the reference tree itself:
  * pack_*.npz        quant/quantize.py:71-75 ``pack`` (pure numpy, imported with a
                      stand-in mlx module).
  * qmv_*.npz         engine/kernels.py:132-184 ``qmv_multi`` Metal source, compiled
                      for the CPU by oracle/ref_build.py (32 lockstep host threads per
                      simdgroup).
  * gd_*.npz          engine/kernels.py:11-75 gated-DeltaNet Metal source (with and
                      without the pre-last-step snapshot), same harness.

mx.quantize / mx.quantized_matmul themselves live in MLX 0.32.0, which is not installed
and not vendored: there is no fixture for them (parity unpinned against MLX).

Inputs come from tests/golden/detrand.py so that large tensors need not be stored:
small fixtures store inputs and outputs; the config-3-shaped fixture stores the
outputs, the seeds, and SHA-256 digests of the fp32 states.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(Path(__file__).resolve().parent))

import detrand  # noqa: E402
import oracle as O  # noqa: E402
import ref_build as R  # noqa: E402

OUT = Path(__file__).resolve().parent


def bf(a: np.ndarray) -> np.ndarray:
    return O.f32_to_bf16(np.asarray(a, dtype=np.float32))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def qmv_inputs(M, K, N, seed):
    """Config-0 style: x ~ N(0,1), uniform codes, scales |N(0,1)|*0.002, biases -8*scale."""
    x = bf(detrand.normal((M, K), seed))
    codes = detrand.integers((N, K), seed + 1, 16).astype(np.uint8)
    w = O.pack4(codes)
    s = bf(np.abs(detrand.normal((N, K // 64), seed + 2)) * 0.002)
    b = bf(-8.0 * O.bf16_to_f32(s))
    return x, codes, w, s, b


def gd_inputs(B, T, Hk, Hv, Dk, Dv, seed, state_kind):
    """Config-3 style: L2-normalised q,k, v ~ N(0,1), a,b ~ N(0,1); A_log = dt_bias = 0
    unless the case asks for non-zero gate parameters."""
    def l2n(t):
        return t / np.sqrt((t * t).sum(-1, keepdims=True))
    q = bf(l2n(detrand.normal((B, T, Hk, Dk), seed)))
    k = bf(l2n(detrand.normal((B, T, Hk, Dk), seed + 1)))
    v = bf(detrand.normal((B, T, Hv, Dv), seed + 2))
    a = bf(detrand.normal((B, T, Hv), seed + 3))
    b = bf(detrand.normal((B, T, Hv), seed + 4))
    if state_kind == "zeros":
        st = np.zeros((B, Hv, Dv, Dk), np.float32)
    else:
        st = (detrand.normal((B, Hv, Dv, Dk), seed + 5) * 0.1).astype(np.float32)
    return q, k, v, a, b, st


def main(ref_root: Path) -> None:
    R.build(ref_root)
    kernels, quant = R.import_reference(ref_root)

    # ---- packing (bit order), including the all-0 / all-15 / alternating edges
    codes = detrand.integers((16, 256), 11, 16).astype(np.uint8)
    codes[0] = 0
    codes[1] = 15
    codes[2] = np.tile(np.array([0, 15], np.uint8), 128)
    codes[3] = np.arange(256) % 16
    np.savez_compressed(OUT / "pack_4bit.npz", codes=codes, packed=quant.pack(codes, 4))

    # ---- qmv_multi (M = 1..8, K % 512 == 0 as the reference kernel requires)
    for (M, K, N) in R.QMV_SHAPES:
        x, codes, w, s, b = qmv_inputs(M, K, N, seed=100 + M * 7 + N)
        y = R.ref_qmv_multi(x, w, s, b)
        np.savez_compressed(OUT / f"qmv_m{M}_k{K}_n{N}.npz", x=x, w=w, scales=s, biases=b, y=y)

    # ---- gated delta, small shapes: full inputs/outputs, with and without snapshot
    cases = [(2, 5, 2, 4, 32, 32, "normal", True, True),
             (1, 7, 1, 2, 64, 32, "zeros", False, True),
             (1, 3, 2, 4, 128, 128, "normal", True, False)]
    for (B, T, Hk, Hv, Dk, Dv, sk, mid, gates) in cases:
        q, k, v, a, b, st = gd_inputs(B, T, Hk, Hv, Dk, Dv, 300 + T, sk)
        A_log = (detrand.normal((Hv,), 400) * 0.5).astype(np.float32) if gates else np.zeros(Hv, np.float32)
        dt = (detrand.normal((Hv,), 401) * 0.5).astype(np.float32) if gates else np.zeros(Hv, np.float32)
        outs = R.ref_gated_delta(q, k, v, a, b, A_log, dt, st, keep_mid=mid)
        rec = dict(q=q, k=k, v=v, a=a, b=b, A_log=A_log, dt_bias=dt, state=st, y=outs[0],
                   state_out=outs[1])
        if mid:
            rec["state_mid"] = outs[2]
        np.savez_compressed(OUT / f"gd_b{B}_t{T}_hk{Hk}_hv{Hv}_dk{Dk}_dv{Dv}{'_mid' if mid else ''}.npz", **rec)

    # ---- gated delta at the Qwen3.5-9B linear-attention shape (Hk=16, Hv=32, D=128),
    # 4 steps with the snapshot (the rollback case), inputs regenerated from seeds.
    for sk in ("zeros", "normal"):
        B, T, Hk, Hv, Dk, Dv = 1, 4, 16, 32, 128, 128
        seed = 500 if sk == "zeros" else 600
        q, k, v, a, b, st = gd_inputs(B, T, Hk, Hv, Dk, Dv, seed, sk)
        A_log = np.zeros(Hv, np.float32)
        dt = np.zeros(Hv, np.float32)
        y, so, sm = R.ref_gated_delta(q, k, v, a, b, A_log, dt, st, keep_mid=True)
        np.savez_compressed(OUT / f"gd_qwen35_t4_{sk}.npz", seed=np.int64(seed), state_kind=sk,
                            y=y, state_out_sha=sha(so), state_mid_sha=sha(sm),
                            state_out_sample=so.reshape(-1)[::4099].copy(),
                            state_mid_sample=sm.reshape(-1)[::4099].copy())
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else R.DEFAULT_REF)
