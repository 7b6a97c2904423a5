"""Generates ref_primitives.npz: golden input/output vectors of the
reference's own functions, compiled from its sources into
oracle/_ref/libref.so (`make -C oracle` where the reference sources are
present). The fixture pins the oracle without the reference at test time.

    python tests/golden/make_golden.py

Functions and files they come from (reference source tree):
  quantize_to_uint8      dequantized_tensor.c:112-143
  dot_product_u8_i8      dequantized_tensor.c:149-196 (one 32-byte block)
  matmul_dequantized     dequantized_tensor.c:204-283 (per-row scale mode)
  rms_norm_avx2          activations_avx2.c:108-143
  swiglu_avx2 / silu     activations_avx2.c:86-105, 33-63
  apply_rope             inference.c:159-190 (theta as a parameter)
  compute_attention      inference.c:193-247
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import bind  # noqa: E402


def main():
    ref = bind.Ref()
    rng = np.random.default_rng(20261201)
    out = {}
    # activation quantisation: rounding ties, clamps, NaN / inf / out of int32 range
    x = (rng.standard_normal(4096) * 2.0).astype(np.float32)
    special = np.array([0.5 / 127, -0.5 / 127, 1.5 / 127, 2.5 / 127, -128.5 / 127, 127.5 / 127, 1.0, -1.0,
                        np.nan, np.inf, -np.inf, 1e30, -1e30, 2.0e7, -2.0e7, 0.0, -0.0], np.float32)
    x[: special.size] = special
    out["quant_x"], out["quant_q"] = x, ref.quant_u8(x)
    # per-32-block dots, [-8,7] weights and (q-8)*16 weights (int16 pair saturation)
    a = rng.integers(0, 256, (6, 3072), dtype=np.uint8)
    q = rng.integers(0, 16, (6, 3072)) - 8
    w = np.concatenate([q[:3], np.clip(q[3:] * 16, -128, 127)]).astype(np.int8)
    dots = np.array([[ref.dot(np.ascontiguousarray(a[i, 32 * b:32 * b + 32]),
                              np.ascontiguousarray(w[i, 32 * b:32 * b + 32])) for b in range(96)]
                     for i in range(6)], np.int32)
    out["dots_a"], out["dots_w"], out["dots"] = a, w, dots
    # matmul_dequantized, per-row scale
    A = rng.standard_normal((3, 3072)).astype(np.float32)
    W = np.clip((rng.integers(0, 16, (24, 3072)) - 8) * 16, -128, 127).astype(np.int8)
    s = (rng.random(24) * 0.01 + 1e-4).astype(np.float32)
    out["mm_A"], out["mm_W"], out["mm_s"], out["mm_C"] = A, W, s, ref.matmul_dequantized(A, W, s)
    # rms_norm, swiglu, silu
    xr = (rng.standard_normal(3072) * 7.0).astype(np.float32)
    out["rms_x"], out["rms_y"] = xr, ref.rms_norm(xr)
    g = (rng.standard_normal(1024) * 3).astype(np.float32)
    u = rng.standard_normal(1024).astype(np.float32)
    out["swiglu_g"], out["swiglu_u"], out["swiglu_y"] = g, u, ref.swiglu(g, u)
    out["silu_y"] = ref.silu(g)
    # RoPE (seq 5, 4 query heads, 2 KV heads, hd 96) at theta 10000
    seq, H, Hk, hd = 5, 4, 2, 96
    rq = rng.standard_normal((seq, H * hd)).astype(np.float32)
    rk = rng.standard_normal((seq, Hk * hd)).astype(np.float32)
    oq, ok = ref.apply_rope(rq, rk, seq, H, Hk, hd, 10000.0)
    out["rope_q"], out["rope_k"], out["rope_oq"], out["rope_ok"] = rq, rk, oq, ok
    # causal GQA attention (seq 7, 4 heads, 2 KV heads, hd 32)
    seq, H, Hk, hd = 7, 4, 2, 32
    Q = rng.standard_normal((seq, H * hd)).astype(np.float32)
    K = rng.standard_normal((seq, Hk * hd)).astype(np.float32)
    V = rng.standard_normal((seq, Hk * hd)).astype(np.float32)
    out["attn_Q"], out["attn_K"], out["attn_V"] = Q, K, V
    out["attn_O"] = ref.compute_attention(Q, K, V, seq, H, Hk, hd)
    np.savez_compressed(os.path.join(HERE, "ref_primitives.npz"), **out)
    print("wrote", os.path.join(HERE, "ref_primitives.npz"))


if __name__ == "__main__":
    main()
