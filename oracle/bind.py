"""ctypes binding of the CPU oracle -- TEST INFRASTRUCTURE.

Loads oracle/liboracle.so (the restatement) and, when present,
oracle/_ref/libref.so (the reference's own sources compiled in place). Only
tests/, the smoke() check and bench.py's CPU-baseline leg import this; the
product library never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref.so")

VP, I, F = C.c_void_p, C.c_int, C.c_float


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class Dims(C.Structure):
    _fields_ = [("vocab", I), ("d", I), ("ffn", I), ("layers", I), ("heads", I), ("kv_heads", I),
                ("head_dim", I), ("theta", F), ("eps", F)]


class Lin(C.Structure):
    _fields_ = [("w", VP), ("s", VP), ("N", I), ("K", I), ("f32", VP), ("wp", VP), ("sp", VP)]


class Layer(C.Structure):
    _fields_ = [(n, Lin) for n in ("q", "k", "v", "o", "gate", "up", "down")]


class Model(C.Structure):
    _fields_ = [("dims", Dims), ("embed", VP), ("base", C.POINTER(Layer)), ("draft_layers", I),
                ("draft", C.POINTER(Layer)), ("lm", Lin), ("n_medusa", I), ("medusa", C.POINTER(Lin))]


class KV(C.Structure):
    _fields_ = [("k", VP), ("v", VP), ("layers", I), ("cap", I), ("kv_heads", I), ("head_dim", I)]


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise RuntimeError(f"{path} missing: make -C oracle")
        self.so = C.CDLL(path)
        s = self.so
        s.orc_dot_pairsat.restype = C.c_int32
        s.orc_dot_plain.restype = C.c_int32
        s.orc_fast_sigmoid.restype = F
        s.orc_fast_sigmoid.argtypes = [F]
        s.orc_rmsnorm.argtypes = [VP, VP, I, F]
        s.orc_rope_vec.argtypes = [VP, I, I, I, F]
        s.orc_f16_to_f32.restype = F
        s.orc_f16_to_f32.argtypes = [C.c_uint16]
        s.orc_f32_to_f16.restype = C.c_uint16
        s.orc_f32_to_f16.argtypes = [F]
        s.orc_argmax.restype = I
        s.orc_spec_generate.restype = I
        s.orc_kv_init.restype = I
        s.orc_stack_forward.argtypes = [C.POINTER(Model), C.POINTER(Layer), I, C.POINTER(KV), VP, I, I, VP, VP]
        s.orc_lm_logits.argtypes = [C.POINTER(Model), VP, VP, I]
        s.orc_kv_init.argtypes = [C.POINTER(KV), I, I, I, I]
        s.orc_kv_free.argtypes = [C.POINTER(KV)]
        s.orc_spec_generate.argtypes = [C.POINTER(Model), VP, I, I, I, I, VP, VP, VP]
        s.orc_greedy_generate.argtypes = [C.POINTER(Model), VP, I, I, VP, VP]
        s.orc_philox_uniform.restype = C.c_float
        s.orc_philox_uniform.argtypes = [C.c_uint32] * 5
        s.orc_philox_u24.restype = C.c_uint32
        s.orc_philox_u24.argtypes = [C.c_uint32] * 5
        s.orc_sample_dist.argtypes = [VP, I, C.c_float, C.c_float, VP]
        s.orc_sample_weight.restype = C.c_uint32
        s.orc_sample_weight.argtypes = [C.c_float]
        s.orc_sample_weights.restype = C.c_uint64
        s.orc_sample_weights.argtypes = [VP, I, C.c_float, C.c_float, VP]
        s.orc_sample_pick.restype = I
        s.orc_sample_pick.argtypes = [VP, VP, I, C.c_uint64, C.c_uint32]
        s.orc_sample_accept.restype = I
        s.orc_sample_accept.argtypes = [C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint64]
        s.orc_sample_residual.restype = C.c_uint64
        s.orc_sample_residual.argtypes = [VP, C.c_uint64, VP, C.c_uint64, I, VP]
        s.orc_spec_generate_sampled.restype = I
        s.orc_spec_generate_sampled.argtypes = [C.POINTER(Model), VP, I, I, I, C.c_float, C.c_float, C.c_uint32,
                                                C.c_uint32, VP, VP]
        s.orc_medusa_generate.restype = I
        s.orc_medusa_generate.argtypes = [C.POINTER(Model), VP, I, VP, I, I, VP, VP, VP]
        s.orc_medusa_tree.restype = I
        s.orc_medusa_tree.argtypes = [I, I, VP, VP, VP, I, I, VP, VP, VP, VP]
        # Every pointer argument must be declared: an undeclared Python int is
        # passed as a 32-bit C int and truncates heap addresses.
        s.orc_quant_u8.argtypes = [VP, VP, I]
        s.orc_dot_pairsat.argtypes = [VP, VP, I]
        s.orc_dot_plain.argtypes = [VP, VP, I]
        s.orc_matmul_rowscale.argtypes = [VP, VP, VP, VP, I, I, I]
        s.orc_matmul_block.argtypes = [VP, VP, VP, VP, I, I, I]
        s.orc_block_dots.argtypes = [VP, VP, VP, I, I, I]
        s.orc_swiglu.argtypes = [VP, VP, VP, I]
        s.orc_silu.argtypes = [VP, VP, I]
        s.orc_q4_0_quantize_i8.argtypes = [VP, I, VP, VP]
        s.orc_philox4x32_10.argtypes = [VP, VP, VP]
        s.orc_argmax.argtypes = [VP, I]
        s.orc_synth_q4_0_i8.restype = I
        s.orc_synth_q4_0_i8.argtypes = [C.c_uint64, C.c_uint32, I, I, C.c_float, VP, VP]
        s.orc_synth_q4_0_f32.restype = I
        s.orc_synth_q4_0_f32.argtypes = [C.c_uint64, C.c_uint32, I, I, C.c_float, VP]
        s.orc_pack_rows8.argtypes = [VP, VP, I, I, VP, VP]
        s.orc_matmul_packed.argtypes = [VP, VP, VP, VP, I, I, I]
        s.orc_last_decode_seconds.restype = C.c_double

    # ----------------------------------------------------------- primitives
    def quant_u8(self, x):
        x = np.ascontiguousarray(x, np.float32)
        q = np.empty(x.shape, np.uint8)
        self.so.orc_quant_u8(_p(x), _p(q), x.size)
        return q

    def dot_pairsat(self, a, w):
        return self.so.orc_dot_pairsat(_p(a), _p(w), a.size)

    def matmul_rowscale(self, A, W, s):
        M, K = A.shape
        N = W.shape[0]
        Cm = np.empty((M, N), np.float32)
        self.so.orc_matmul_rowscale(_p(A), _p(W), _p(s), _p(Cm), M, N, K)
        return Cm

    def matmul_block(self, A, W, d):
        A = np.ascontiguousarray(A, np.float32)
        M, K = A.shape
        N = W.shape[0]
        Cm = np.empty((M, N), np.float32)
        self.so.orc_matmul_block(_p(A), _p(W), _p(d), _p(Cm), M, N, K)
        return Cm

    def pack_rows8(self, W, d):
        """orc_pack_rows8: (wp, sp), or None when W is not packable."""
        W = np.ascontiguousarray(W, np.int8)
        d = np.ascontiguousarray(d, np.uint16)
        wp = np.empty_like(W)
        sp = np.empty(d.shape, np.float32)
        if self.so.orc_pack_rows8(_p(W), _p(d), W.shape[0], W.shape[1], _p(wp), _p(sp)) != 0:
            return None
        return wp, sp

    def matmul_packed(self, A, wp, sp):
        A = np.ascontiguousarray(A, np.float32)
        M, K = A.shape
        N = wp.shape[0]
        Cm = np.empty((M, N), np.float32)
        self.so.orc_matmul_packed(_p(A), _p(wp), _p(sp), _p(Cm), M, N, K)
        return Cm

    def block_dots(self, A, W):
        A = np.ascontiguousarray(A, np.float32)
        M, K = A.shape
        N = W.shape[0]
        D = np.empty((M, N, K // 32), np.int32)
        self.so.orc_block_dots(_p(A), _p(W), _p(D), M, N, K)
        return D

    def rmsnorm(self, x, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        o = np.empty_like(x)
        self.so.orc_rmsnorm(_p(x), _p(o), x.size, eps)
        return o

    def swiglu(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        o = np.empty_like(g)
        self.so.orc_swiglu(_p(g), _p(u), _p(o), g.size)
        return o

    def silu(self, x):
        x = np.ascontiguousarray(x, np.float32)
        o = np.empty_like(x)
        self.so.orc_silu(_p(x), _p(o), x.size)
        return o

    def rope_vec(self, v, heads, head_dim, pos, theta):
        v = np.array(v, np.float32, copy=True)
        self.so.orc_rope_vec(_p(v), heads, head_dim, pos, theta)
        return v

    def synth_q4_0_i8(self, seed, tid, rows, cols, std=0.02):
        w = np.empty((rows, cols), np.int8)
        d = np.empty((rows, cols // 32), np.uint16)
        assert self.so.orc_synth_q4_0_i8(seed, tid, rows, cols, std, _p(w), _p(d)) == 0
        return w, d

    def synth_q4_0_f32(self, seed, tid, rows, cols, std=0.02):
        o = np.empty((rows, cols), np.float32)
        assert self.so.orc_synth_q4_0_f32(seed, tid, rows, cols, std, _p(o)) == 0
        return o

    def q4_0_i8(self, x):
        x = np.ascontiguousarray(x, np.float32)
        w = np.empty(x.size, np.int8)
        d = np.empty(x.size // 32, np.uint16)
        self.so.orc_q4_0_quantize_i8(_p(x), x.size, _p(w), _p(d))
        return w, d

    def sample_dist(self, logits, T, top_p):
        lg = np.ascontiguousarray(logits, np.float32)
        q = np.empty_like(lg)
        self.so.orc_sample_dist(_p(lg), lg.size, T, top_p, _p(q))
        return q

    def sample_weights(self, logits, T, top_p):
        """(E uint32 nucleus weights, kept mass M)."""
        lg = np.ascontiguousarray(logits, np.float32)
        E = np.empty(lg.size, np.uint32)
        M = self.so.orc_sample_weights(_p(lg), lg.size, T, top_p, _p(E))
        return E, int(M)

    def sample_weight(self, x):
        return int(self.so.orc_sample_weight(float(x)))

    def sample_pick(self, w, total, U):
        """Inverse-CDF pick over integer weights (uint32 or uint64) at U / 2^24."""
        if w.dtype == np.uint32:
            w = np.ascontiguousarray(w)
            return self.so.orc_sample_pick(_p(w), None, w.size, int(total), int(U))
        w = np.ascontiguousarray(w, np.uint64)
        return self.so.orc_sample_pick(None, _p(w), w.size, int(total), int(U))

    def sample_accept(self, U, Ep, Mp, Eq, Mq):
        return bool(self.so.orc_sample_accept(int(U), int(Ep), int(Mp), int(Eq), int(Mq)))

    def sample_residual(self, Ep, Mp, Eq, Mq):
        Ep = np.ascontiguousarray(Ep, np.uint32)
        Eq = np.ascontiguousarray(Eq, np.uint32)
        R = np.empty(Ep.size, np.uint64)
        s = self.so.orc_sample_residual(_p(Ep), int(Mp), _p(Eq), int(Mq), Ep.size, _p(R))
        return R, int(s)

    def philox_u24(self, seed, seq, step, pos, purpose):
        return int(self.so.orc_philox_u24(seed & 0xFFFFFFFF, seq, step & 0xFFFFFFFF, pos, purpose))

    def philox(self, ctr, key):
        c = np.asarray(ctr, np.uint32)
        k = np.asarray(key, np.uint32)
        o = np.empty(4, np.uint32)
        self.so.orc_philox4x32_10(_p(c), _p(k), _p(o))
        return o


class OracleModel:
    """Oracle model over numpy weights. `w` maps (stack, layer, proj) to
    (int8 [N,K], fp16 bits [N,K/32]); stack 3 proj 1 = LM head."""

    def __init__(self, orc: Oracle, dims: dict, embed, w, draft_layers=0, n_medusa=0, f32=None, packed=False):
        self.orc = orc
        self.keep = [embed]
        self.m = Model()
        D = self.m.dims
        for k in ("vocab", "d", "ffn", "layers", "heads", "kv_heads", "head_dim", "theta", "eps"):
            setattr(D, k, dims[k])
        self.m.embed = _p(embed)

        def lin(key):
            L = Lin()
            if f32 is not None and key in f32:
                a = np.ascontiguousarray(f32[key], np.float32)
                self.keep.append(a)
                L.f32 = _p(a)
                L.N, L.K = a.shape
                return L
            wq, dq = w[key]
            if packed and wq.shape[0] % 8 == 0:
                # weights repacked for 8-lane integer dots (orc_pack_rows8);
                # same results, the reference kernel's speed
                wp = np.empty_like(wq)
                sp = np.empty(dq.shape, np.float32)
                if orc.so.orc_pack_rows8(_p(wq), _p(dq), wq.shape[0], wq.shape[1], _p(wp), _p(sp)) == 0:
                    self.keep += [wp, sp]
                    L.wp, L.sp = _p(wp), _p(sp)
                    L.N, L.K = wq.shape
                    return L
            wq, dq = w[key]
            self.keep += [wq, dq]
            L.w, L.s = _p(wq), _p(dq)
            L.N, L.K = wq.shape
            return L

        def stack(s, n):
            arr = (Layer * max(n, 1))()
            for l in range(n):
                for pi, name in enumerate(("q", "k", "v", "o", "gate", "up", "down")):
                    setattr(arr[l], name, lin((s, l, pi)))
            self.keep.append(arr)
            return arr

        self.m.base = stack(0, dims["layers"])
        self.m.draft_layers = draft_layers
        self.m.draft = stack(1, draft_layers)
        self.m.lm = lin((3, 0, 1))
        self.m.n_medusa = n_medusa
        med = (Lin * max(n_medusa, 1))()
        for h in range(n_medusa):
            med[h] = lin((2, h, 0))
        self.keep.append(med)
        self.m.medusa = med

    def kv(self, layers, cap):
        kv = KV()
        self.orc.so.orc_kv_init(C.byref(kv), layers, cap, self.m.dims.kv_heads, self.m.dims.head_dim)
        return kv

    def stack_forward(self, stack, kv, x, base, pos, mask=None):
        x = np.array(x, np.float32, copy=True)
        pos = np.ascontiguousarray(pos, np.int32)
        mk = None if mask is None else np.ascontiguousarray(mask, np.uint8)
        layers = self.m.base if stack == 0 else self.m.draft
        n = self.m.dims.layers if stack == 0 else self.m.draft_layers
        self.orc.so.orc_stack_forward(C.byref(self.m), layers, n, C.byref(kv), _p(x), x.shape[0], base, _p(pos),
                                      _p(mk))
        return x

    def lm_logits(self, x):
        x = np.ascontiguousarray(x, np.float32)
        lg = np.empty((x.shape[0], self.m.dims.vocab), np.float32)
        self.orc.so.orc_lm_logits(C.byref(self.m), _p(x), _p(lg), x.shape[0])
        return lg

    def greedy(self, prompt, n_new):
        p = np.ascontiguousarray(prompt, np.int32)
        o = np.empty(n_new, np.int32)
        mg = np.empty(n_new, np.float32)
        self.orc.so.orc_greedy_generate(C.byref(self.m), _p(p), len(p), n_new, _p(o), _p(mg))
        return o, mg

    def spec(self, prompt, n_new, k, max_acc=None):
        p = np.ascontiguousarray(prompt, np.int32)
        o = np.empty(n_new, np.int32)
        acc = np.zeros(n_new + 1, np.int32)
        mg = np.empty(n_new, np.float32)
        steps = self.orc.so.orc_spec_generate(C.byref(self.m), _p(p), len(p), k, k if max_acc is None else max_acc,
                                              n_new, _p(o), _p(acc), _p(mg))
        return o, acc[:steps], mg


    def spec_sampled(self, prompt, n_new, k, T, top_p, seed, seq_id=0):
        """Stochastic speculative decoding: (tokens, accepted per step)."""
        p = np.ascontiguousarray(prompt, np.int32)
        o = np.empty(n_new, np.int32)
        acc = np.zeros(n_new + 1, np.int32)
        steps = self.orc.so.orc_spec_generate_sampled(C.byref(self.m), _p(p), len(p), k, n_new, T, top_p, seed,
                                                      seq_id, _p(o), _p(acc))
        return o, acc[:steps]

    def medusa(self, prompt, n_new, topk, max_nodes):
        """Medusa greedy decoding: (tokens, accepted per step, margins)."""
        p = np.ascontiguousarray(prompt, np.int32)
        tk = np.ascontiguousarray(topk, np.int32)
        o = np.empty(n_new, np.int32)
        acc = np.zeros(n_new + 1, np.int32)
        mg = np.empty(n_new, np.float32)
        steps = self.orc.so.orc_medusa_generate(C.byref(self.m), _p(p), len(p), _p(tk), max_nodes, n_new, _p(o),
                                                _p(acc), _p(mg))
        return o, acc[:steps], mg


def medusa_tree(orc, root, topk, tok, prob, max_nodes):
    """orc_medusa_tree: (tokens, parents, depths, scores) of the kept nodes."""
    tk = np.ascontiguousarray(topk, np.int32)
    kmax = tok.shape[1]
    t = np.ascontiguousarray(tok, np.int32)
    pr = np.ascontiguousarray(prob, np.float32)
    ot, op, od = (np.empty(max_nodes, np.int32) for _ in range(3))
    osc = np.empty(max_nodes, np.float32)
    n = orc.so.orc_medusa_tree(root, len(tk), _p(tk), _p(t), _p(pr), kmax, max_nodes, _p(ot), _p(op), _p(od), _p(osc))
    return ot[:n], op[:n], od[:n], osc[:n]


class Ref:
    """The reference's own functions (oracle/_ref/libref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise RuntimeError(f"{path} missing: make -C oracle (needs the reference sources)")
        self.so = C.CDLL(path)
        s = self.so
        s.ref_dot_product_u8_i8.restype = C.c_int32
        s.ref_dot_product_u8_i8.argtypes = [VP, VP, I]
        s.ref_quantize_to_uint8.argtypes = [VP, VP, I]
        s.ref_matmul_dequantized.argtypes = [VP, VP, VP, VP, I, I, I]
        s.ref_rms_norm.argtypes = [VP, VP, I, F]
        s.ref_swiglu.argtypes = [VP, VP, VP, I]
        s.ref_silu.argtypes = [VP, VP, I]
        s.ref_apply_rope.argtypes = [VP, VP, I, I, I, I, F]
        s.ref_compute_attention.argtypes = [VP, VP, VP, VP, I, I, I, I]
        s.ref_model_forward_f32.restype = I
        s.ref_model_forward_f32.argtypes = [I, I, I, I, I, I, I, VP, VP, VP, VP, I, VP]

    def quant_u8(self, x):
        x = np.ascontiguousarray(x, np.float32)
        q = np.empty(x.shape, np.uint8)
        self.so.ref_quantize_to_uint8(_p(x), _p(q), x.size)
        return q

    def dot(self, a, w):
        return self.so.ref_dot_product_u8_i8(_p(a), _p(w), a.size)

    def matmul_dequantized(self, A, W, s):
        A = np.ascontiguousarray(A, np.float32)
        M, K = A.shape
        N = W.shape[0]
        Cm = np.empty((M, N), np.float32)
        self.so.ref_matmul_dequantized(_p(A), _p(W), _p(s), _p(Cm), M, N, K)
        return Cm

    def rms_norm(self, x, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        o = np.empty_like(x)
        self.so.ref_rms_norm(_p(x), _p(o), x.size, eps)
        return o

    def swiglu(self, g, u):
        o = np.empty_like(g)
        self.so.ref_swiglu(_p(g), _p(u), _p(o), g.size)
        return o

    def silu(self, x):
        o = np.empty_like(x)
        self.so.ref_silu(_p(x), _p(o), x.size)
        return o

    def apply_rope(self, q, k, seq, heads, kv_heads, hd, theta):
        q = np.array(q, np.float32, copy=True)
        k = np.array(k, np.float32, copy=True)
        self.so.ref_apply_rope(_p(q), _p(k), seq, heads, kv_heads, hd, theta)
        return q, k

    def compute_attention(self, Q, K, V, seq, heads, kv_heads, hd):
        Q = np.array(Q, np.float32, copy=True)
        K = np.array(K, np.float32, copy=True)
        V = np.ascontiguousarray(V, np.float32)
        out = np.empty((seq, heads * hd), np.float32)
        self.so.ref_compute_attention(_p(Q), _p(K), _p(V), _p(out), seq, heads, kv_heads, hd)
        return out

    def model_forward_f32(self, dims, embed, layers_w, lm, tokens):
        """layers_w: list of 7-tuples of f32 [out, in] arrays per layer."""
        ptrs = (VP * (7 * len(layers_w)))()
        keep = []
        for l, lw in enumerate(layers_w):
            for j, a in enumerate(lw):
                a = np.ascontiguousarray(a, np.float32)
                keep.append(a)
                ptrs[7 * l + j] = _p(a)
        toks = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(dims["vocab"], np.float32)
        tok = self.so.ref_model_forward_f32(dims["vocab"], dims["d"], dims["ffn"], len(layers_w), dims["heads"],
                                            dims["kv_heads"], dims["head_dim"], VP(_p(embed)), ptrs, VP(_p(lm)),
                                            VP(_p(toks)), len(toks), VP(_p(logits)))
        return tok, logits
