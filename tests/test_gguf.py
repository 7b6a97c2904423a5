"""GGUF files with Q4_0 weights (the 18-byte block with an fp16 scale; low
nibbles are elements 0..15, gguf_loader.c:147-161): the loaders turn each
tensor into the same INT8 q-8 values and fp16 block scales the seeded
generator produces, fused attn_qkv / gate+up ffn_up tensors split, and a
device engine loaded from files decodes exactly like one loaded tensor by
tensor."""
import ctypes as C
import os

import numpy as np
import pytest

import flb200
from _gguf import write_gguf
from _model import SMALL, SMALL_GQA, engine_cfg, load_engine, make_weights, prompt

NAMES = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]


def base_tensors(w, embed, dims, stack=0, fused=False):
    out = [("token_embd.weight", "f32", embed), ("output.weight", "q4_0", w[(3, 0, 1)])]
    n = dims["layers"] if stack == 0 else 1
    for l in range(n):
        if fused:
            qkv = [w[(stack, l, p)] for p in range(3)]
            out.append((f"blk.{l}.attn_qkv.weight", "q4_0", (np.concatenate([t[0] for t in qkv]),
                                                              np.concatenate([t[1] for t in qkv]))))
            out.append((f"blk.{l}.attn_output.weight", "q4_0", w[(stack, l, 3)]))
            gu = [w[(stack, l, 4)], w[(stack, l, 5)]]
            out.append((f"blk.{l}.ffn_up.weight", "q4_0", (np.concatenate([t[0] for t in gu]),
                                                           np.concatenate([t[1] for t in gu]))))
            out.append((f"blk.{l}.ffn_down.weight", "q4_0", w[(stack, l, 6)]))
        else:
            for p, nm in enumerate(NAMES):
                out.append((f"blk.{l}.{nm}.weight", "q4_0", w[(stack, l, p)]))
        out.append((f"blk.{l}.attn_norm.weight", "f32", np.ones((1, dims["d"]), np.float32)))
    return out


def host_tensor(t):
    n = t.rows * t.cols
    w = np.ctypeslib.as_array(t.weights, shape=(n,)).reshape(t.rows, t.cols).copy()
    d = np.ctypeslib.as_array(t.scales_f16, shape=(n // 32,)).reshape(t.rows, t.cols // 32).copy()
    return w, d


def test_draft_model_load_gguf(lib, tmp_path):
    """A one-layer draft with fused attn_qkv and Phi-3's fused gate+up:
    the draft's host tensors equal the generator's INT8 and scales."""
    dims = SMALL
    w = {}
    shapes = [(dims["d"], dims["d"])] * 4 + [(dims["ffn"], dims["d"])] * 2 + [(dims["d"], dims["ffn"])]
    for p, (r, c) in enumerate(shapes):
        w[(1, 0, p)] = lib.synth_q4_0_i8(5, flb200.tensor_id(1, 0, p), r, c)
    w[(3, 0, 1)] = lib.synth_q4_0_i8(5, flb200.tensor_id(3, 0, 1), dims["vocab"], dims["d"])
    embed = lib.synth_q4_0_f32(5, flb200.tensor_id(3, 0, 0), dims["vocab"], dims["d"])
    path = str(tmp_path / "draft.gguf")
    write_gguf(path, base_tensors(w, embed, dims, stack=1, fused=True))
    dm = lib.draft_model_create(1, dims["d"], dims["ffn"], dims["vocab"])
    assert lib.draft_model_load(dm, path.encode()) == 0, lib.err()
    m = dm.contents
    for p, arr in enumerate((m.w_q_proj, m.w_k_proj, m.w_v_proj, m.w_o_proj, m.w_gate, m.w_up, m.w_down)):
        got = host_tensor(arr[0])
        assert np.array_equal(got[0], w[(1, 0, p)][0]) and np.array_equal(got[1], w[(1, 0, p)][1]), p
    got = host_tensor(m.w_lm_head[0])
    assert np.array_equal(got[0], w[(3, 0, 1)][0])
    lib.draft_model_free(dm)


def test_gguf_rejects_bad_files(lib, tmp_path):
    dm = lib.draft_model_create(1, 512, 1024, 1000)
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + b"\0" * 64)
    assert lib.draft_model_load(dm, str(bad).encode()) == -1
    assert "magic" in lib.err()
    w = lib.synth_q4_0_i8(1, 1, 64, 512)
    good = tmp_path / "short.gguf"
    write_gguf(str(good), [("blk.0.attn_q.weight", "q4_0", w)])
    good.write_bytes(good.read_bytes()[:-100])
    assert lib.draft_model_load(dm, str(good).encode()) == -1
    assert lib.draft_model_load(dm, str(tmp_path / "missing.gguf").encode()) == -1
    lib.draft_model_free(dm)


@pytest.mark.gpu
@pytest.mark.parametrize("dims", [SMALL, SMALL_GQA], ids=["mha", "gqa"])
def test_engine_from_gguf_decodes_like_tensor_loads(gpu, tmp_path, dims):
    w, embed = make_weights(gpu, dims, seed=17)
    base = str(tmp_path / "base.gguf")
    draft = str(tmp_path / "draft.gguf")
    write_gguf(base, base_tensors(w, embed, dims, stack=0))
    write_gguf(draft, base_tensors(w, embed, dims, stack=1, fused=dims["kv_heads"] == dims["heads"]))
    ref = flb200.Engine(gpu, engine_cfg(dims))
    load_engine(ref, w, embed)
    eng = flb200.Engine(gpu, engine_cfg(dims))
    assert gpu.fl_engine_load_gguf(eng.h, 0, base.encode()) == 0, gpu.err()
    assert gpu.fl_engine_load_gguf(eng.h, 1, draft.encode()) == 0, gpu.err()
    x = embed[prompt(3, 12, dims["vocab"])]
    _, lg0 = ref.forward_rows(0, x, 0, np.arange(12))
    _, lg1 = eng.forward_rows(0, x, 0, np.arange(12))
    assert np.array_equal(lg0, lg1)
    p = prompt(4, 16, dims["vocab"])
    t0, a0 = ref.spec_generate(p, 24, 4)
    t1, a1 = eng.spec_generate(p, 24, 4)
    assert np.array_equal(t0, t1) and np.array_equal(a0, a1)
    ref.close()
    eng.close()
