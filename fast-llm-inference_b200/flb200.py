"""ctypes binding of libfl_b200.so (include/*.h) for Python callers.

The library is the product: C ABI, sm_100a kernels, no Python compute. This
module only declares the signatures and offers numpy conveniences. Loading
fails loudly when the shared library is missing; there is no fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfl_b200.so")

FL_OK = 0


class FLError(RuntimeError):
    pass


class DequantizedTensor(C.Structure):
    """dequantized_tensor_t (include/dequantized_tensor.h)."""
    _fields_ = [
        ("weights", C.POINTER(C.c_int8)),
        ("scales", C.POINTER(C.c_float)),
        ("f32_weights", C.POINTER(C.c_float)),
        ("rows", C.c_int),
        ("cols", C.c_int),
        ("original_bits", C.c_int),
        ("scale_block", C.c_int),
        ("scales_f16", C.POINTER(C.c_uint16)),
        ("dev", C.c_void_p),
    ]


class ModelConfig(C.Structure):
    """fl_model_config_t (include/fl_cuda.h)."""
    _fields_ = [
        ("vocab_size", C.c_int),
        ("hidden_size", C.c_int),
        ("intermediate_size", C.c_int),
        ("num_layers", C.c_int),
        ("num_heads", C.c_int),
        ("num_kv_heads", C.c_int),
        ("head_dim", C.c_int),
        ("draft_layers", C.c_int),
        ("medusa_heads", C.c_int),
        ("max_seq_len", C.c_int),
        ("rope_theta", C.c_float),
        ("norm_eps", C.c_float),
    ]


class MedusaConfig(C.Structure):
    """medusa_config_t"""
    _fields_ = [("num_heads", C.c_int), ("top_k", C.c_int), ("temperature", C.c_float)]


class MedusaTree(C.Structure):
    """medusa_tree_t"""
    _fields_ = [("tokens", C.POINTER(C.c_int)), ("probs", C.POINTER(C.c_float)),
                ("parent_indices", C.POINTER(C.c_int)), ("positions", C.POINTER(C.c_int)),
                ("num_candidates", C.c_int), ("max_candidates", C.c_int)]


class SpecConfig(C.Structure):
    """speculative_config_t (include/speculative.h)."""
    _fields_ = [("num_draft_tokens", C.c_int), ("temperature", C.c_float), ("max_accepted", C.c_int)]


class DraftTree(C.Structure):
    _fields_ = [("tokens", C.POINTER(C.c_int)), ("probs", C.POINTER(C.c_float)),
                ("num_tokens", C.c_int), ("max_tokens", C.c_int)]


class DraftKV(C.Structure):
    _fields_ = [("k_cache", C.POINTER(C.c_float)), ("v_cache", C.POINTER(C.c_float)),
                ("cache_len", C.c_int), ("max_len", C.c_int)]


class DraftModel(C.Structure):
    _fields_ = [(n, C.POINTER(DequantizedTensor)) for n in
                ("w_q_proj", "w_k_proj", "w_v_proj", "w_o_proj", "w_gate", "w_up", "w_down", "w_lm_head")] + \
               [("num_layers", C.c_int), ("hidden_size", C.c_int), ("intermediate_size", C.c_int),
                ("vocab_size", C.c_int)]


VP = C.c_void_p
I = C.c_int
F = C.c_float
U64 = C.c_uint64
U32 = C.c_uint32
SZ = C.c_size_t

_SIGS = {
    "fl_cuda_last_error": (C.c_char_p, []),
    "fl_cuda_init": (I, [I]),
    "fl_cuda_device_count": (I, [C.POINTER(I)]),
    "fl_cuda_sync": (I, []),
    "fl_cuda_tp_wait_timeout_check": (I, []),
    "fl_cuda_medusa_tree": (I, [VP, VP, VP, I, I, I, I, I, VP, VP, VP, VP, VP]),
    "fl_cuda_block_dots_w4": (I, [VP, C.POINTER(DequantizedTensor), VP, I, I, I, VP]),
    "fl_engine_set_weight_bits": (I, [VP, I]),
    "fl_argmax_key": (C.c_uint64, [C.c_float, I]),
    "fl_tp_merge_topw": (I, [VP, I, C.c_size_t, I, VP]),
    "fl_engine_draft_lm": (I, [VP, VP, I, I, I, VP]),
    "fl_engine_lm_argmax": (I, [VP, VP, VP]),
    "fl_engine_lm_logits": (I, [VP, VP, VP]),
    "fl_cuda_stream": (VP, []),
    "fl_cuda_malloc": (I, [C.POINTER(VP), SZ]),
    "fl_cuda_free": (I, [VP]),
    "fl_cuda_h2d": (I, [VP, VP, SZ]),
    "fl_cuda_d2h": (I, [VP, VP, SZ]),
    "fl_cuda_memset": (I, [VP, I, SZ]),
    "fl_cuda_upload_tensor": (I, [C.POINTER(DequantizedTensor)]),
    "fl_cuda_act_quant": (I, [VP, VP, I, I, I, F, VP]),
    "fl_cuda_matmul_i8": (I, [VP, C.POINTER(DequantizedTensor), VP, I, I, I, VP]),
    "fl_cuda_gemv_i8": (I, [VP, C.POINTER(DequantizedTensor), VP, I, I, I, VP]),
    "fl_cuda_block_dots_i8": (I, [VP, C.POINTER(DequantizedTensor), VP, I, I, I, VP]),
    "fl_cuda_block_dots_i8_noalloc": (I, [VP, C.POINTER(DequantizedTensor), VP, I, I, I, VP]),
    "fl_synth_q4_0_i8": (I, [U64, U32, I, I, F, VP, VP]),
    "fl_synth_q4_0_i8_block": (I, [U64, U32, I, I, I, I, I, I, F, VP, VP]),
    "fl_synth_q4_0_f32": (I, [U64, U32, I, I, F, VP]),
    "fl_synth_normal": (I, [U64, U32, SZ, F, VP]),
    "fl_q4_0_to_i8": (I, [VP, I, I, VP, VP]),
    "fl_philox4x32_10": (None, [VP, VP, VP]),
    "fl_engine_create": (VP, [C.POINTER(ModelConfig), I]),
    "fl_engine_create_tp": (VP, [C.POINTER(ModelConfig), I, I, I, VP]),
    "fl_engine_tp": (I, [VP, VP, VP]),
    "fl_tp_unique_id": (I, [VP]),
    "fl_tp_layout": (I, [C.POINTER(ModelConfig), I, I, VP]),
    "fl_engine_destroy": (None, [VP]),
    "fl_engine_load_linear": (I, [VP, I, I, I, VP, VP, I, I]),
    "fl_engine_load_embedding": (I, [VP, VP]),
    "fl_engine_load_gguf": (I, [VP, I, C.c_char_p]),
    "fl_engine_dims": (I, [VP, VP]),
    "fl_engine_synthesize": (I, [VP, U64]),
    "fl_engine_ready": (I, [VP]),
    "fl_engine_forward_rows": (I, [VP, I, VP, I, I, VP, VP, VP, VP]),
    "fl_engine_greedy_generate": (I, [VP, VP, I, I, VP]),
    "fl_engine_spec_generate": (I, [VP, VP, I, I, I, I, VP, VP, VP]),
    "fl_engine_spec_prefill": (I, [VP, VP, I, I, I]),
    "fl_engine_spec_decode": (I, [VP, I, VP, VP, VP]),
    "fl_engine_set_sampling": (I, [VP, F, F, U32, U32]),
    "fl_engine_spec_generate_batch": (I, [VP, VP, I, I, VP, I, I, VP, VP]),
    "fl_engine_batch_reserve": (I, [VP, I, I]),
    "fl_engine_batch_capacity": (I, [VP, VP, VP]),
    "fl_engine_batch_prefill": (I, [VP, VP, I, I, VP, I]),
    "fl_engine_batch_begin": (I, [VP, I]),
    "fl_engine_batch_decode": (I, [VP, I, VP, VP]),
    "fl_engine_batch_step": (I, [VP, VP]),
    "fl_engine_batch_trace": (I, [VP, I, VP, VP, VP, VP, VP, VP]),
    "fl_engine_get_sampling": (I, [VP, VP, VP, VP, VP]),
    "fl_engine_sample_trace_enable": (I, [VP, I]),
    "fl_engine_sample_trace": (I, [VP, VP, VP, VP, VP, VP, VP]),
    "fl_engine_spec_begin": (I, [VP, I]),
    "fl_engine_spec_step": (I, [VP, VP]),
    "fl_engine_last_timing": (I, [VP, VP, VP, VP]),
    "fl_engine_stream": (VP, [VP]),
    "fl_engine_last_launches": (C.c_longlong, [VP]),
    "fl_engine_step_kernel": (I, [VP]),
    "fl_engine_step_trace": (I, [VP, VP, VP, I]),
    "fl_engine_step_trace_stages": (I, [VP, VP]),
    "fl_engine_medusa_generate": (I, [VP, VP, I, I, VP, I, I, VP, VP, VP]),
    "fl_engine_spec_medusa_generate": (I, [VP, VP, I, I, I, VP, I, I, VP, VP, VP]),
    "fl_engine_spec_tree_generate": (I, [VP, VP, I, I, I, I, VP, VP, VP]),
    "fl_engine_batch_tree_generate": (I, [VP, VP, I, I, I, I, I, VP, VP]),
    "fl_engine_medusa_tree": (I, [VP, VP, I, VP, I, I, VP, VP, VP, VP]),
    "fl_engine_tree_verify": (I, [VP, VP, VP, VP, I, VP, VP]),
    "fl_engine_bind_medusa": (I, [VP, VP]),
    "fl_engine_draft_bound": (I, [VP, VP]),
    "fl_engine_note_draft": (None, [VP, VP]),
    "fl_engine_bench_linear": (I, [VP, I, I, I, I, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "fl_engine_bench_attention": (I, [VP, I, I, I, I, C.POINTER(C.c_double)]),
    "fl_engine_position": (I, [VP]),
    "fl_engine_set_position": (I, [VP, I]),
    "fl_cuda_base_forward": (None, [VP, VP, I, VP, I]),
    "fl_engine_last_feature": (I, [VP, VP]),
    "fl_engine_draft_chain": (I, [VP, VP, I, I, I, VP, VP]),
    "fl_engine_bind_draft": (I, [VP, VP]),
    "fl_draft_tree_set_vocab": (I, [VP, I]),
    "matmul_dequantized": (None, [VP, C.POINTER(DequantizedTensor), VP, I, I, I]),
    "dequantized_tensor_free": (None, [C.POINTER(DequantizedTensor)]),
    "dequantized_from_q4": (C.POINTER(DequantizedTensor), [VP]),
    "dequantized_from_q8": (C.POINTER(DequantizedTensor), [VP]),
    "draft_model_create": (C.POINTER(DraftModel), [I, I, I, I]),
    "draft_model_load": (I, [C.POINTER(DraftModel), C.c_char_p]),
    "draft_model_free": (None, [C.POINTER(DraftModel)]),
    "draft_tree_create": (C.POINTER(DraftTree), [I]),
    "draft_tree_free": (None, [C.POINTER(DraftTree)]),
    "draft_kv_cache_create": (C.POINTER(DraftKV), [I, I, I]),
    "draft_kv_cache_free": (None, [C.POINTER(DraftKV)]),
    "verify_tokens": (I, [VP, C.POINTER(DraftTree), VP, C.POINTER(I), C.POINTER(SpecConfig)]),
    "speculative_generate": (I, [C.POINTER(DraftModel), VP, VP, VP, I, VP, I, C.POINTER(SpecConfig)]),
    "speculative_decode_step": (I, [C.POINTER(DraftModel), C.POINTER(DraftKV), VP, VP, VP, I, VP, VP,
                                    C.POINTER(SpecConfig)]),
    "medusa_model_create": (VP, [I, I, I]),
    "medusa_model_load": (I, [VP, C.c_char_p]),
    "medusa_model_free": (None, [VP]),
    "medusa_generate": (I, [VP, VP, VP, VP, I, VP, I, C.POINTER(MedusaConfig)]),
    "speculative_medusa_generate": (I, [C.POINTER(DraftModel), VP, VP, VP, VP, VP, I, VP, I, C.POINTER(MedusaConfig)]),
    "fl_medusa_set_tree": (I, [VP, VP, I, I]),
    "medusa_tree_create": (C.POINTER(MedusaTree), [I]),
    "medusa_tree_free": (None, [C.POINTER(MedusaTree)]),
    "medusa_predict": (I, [VP, VP, I, C.POINTER(MedusaTree), C.POINTER(MedusaConfig)]),
    "medusa_build_tree": (I, [VP, VP, C.POINTER(MedusaTree), C.POINTER(MedusaConfig)]),
    "medusa_verify_tree": (I, [VP, VP, C.POINTER(MedusaTree), VP, VP, C.POINTER(MedusaConfig)]),
    "medusa_decode_step": (I, [VP, VP, VP, VP, I, VP, VP, C.POINTER(MedusaConfig)]),
}


def ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the C ABI must be contiguous"
    return a.ctypes.data


class Lib:
    """Loaded libfl_b200.so with typed functions."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise FLError(f"{path} is missing: build it with fast-llm-inference_b200/build.py")
        self.path = path
        self.so = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(self.so, name)
            fn.restype = res
            fn.argtypes = args
            setattr(self, name, fn)

    def err(self) -> str:
        m = self.fl_cuda_last_error()
        return m.decode() if m else ""

    def check(self, rc: int, what: str = "") -> None:
        if rc != FL_OK:
            raise FLError(f"{what} failed ({rc}): {self.err()}")

    def device_count(self) -> int:
        n = C.c_int(0)
        self.fl_cuda_device_count(C.byref(n))
        return n.value

    # --------------------------------------------------------------- synth
    def synth_q4_0_i8(self, seed: int, tid: int, rows: int, cols: int, std: float = 0.02):
        w = np.empty((rows, cols), np.int8)
        d = np.empty((rows, cols // 32), np.uint16)
        self.check(self.fl_synth_q4_0_i8(seed, tid, rows, cols, std, ptr(w), ptr(d)), "synth")
        return w, d

    def synth_q4_0_f32(self, seed: int, tid: int, rows: int, cols: int, std: float = 0.02):
        o = np.empty((rows, cols), np.float32)
        self.check(self.fl_synth_q4_0_f32(seed, tid, rows, cols, std, ptr(o)), "synth")
        return o

    def synth_normal(self, seed: int, tid: int, count: int, std: float = 1.0):
        o = np.empty(count, np.float32)
        self.check(self.fl_synth_normal(seed, tid, count, std, ptr(o)), "synth")
        return o

    def philox(self, ctr, key):
        c = np.asarray(ctr, np.uint32)
        k = np.asarray(key, np.uint32)
        o = np.empty(4, np.uint32)
        self.fl_philox4x32_10(ptr(c), ptr(k), ptr(o))
        return o


def tensor_id(stack: int, layer: int, proj: int) -> int:
    return (stack << 24) | (layer << 8) | proj


def block_tensor(w: np.ndarray, d: np.ndarray) -> DequantizedTensor:
    """Block-mode dequantized_tensor_t over numpy arrays (kept alive by caller)."""
    t = DequantizedTensor()
    t.weights = w.ctypes.data_as(C.POINTER(C.c_int8))
    t.scales = None
    t.f32_weights = None
    t.rows, t.cols = w.shape
    t.original_bits = 4
    t.scale_block = 32
    t.scales_f16 = d.ctypes.data_as(C.POINTER(C.c_uint16))
    t.dev = None
    return t


def row_tensor(w: np.ndarray, s: np.ndarray) -> DequantizedTensor:
    """Per-row-scale dequantized_tensor_t (the reference's own mode)."""
    t = DequantizedTensor()
    t.weights = w.ctypes.data_as(C.POINTER(C.c_int8))
    t.scales = s.ctypes.data_as(C.POINTER(C.c_float))
    t.f32_weights = None
    t.rows, t.cols = w.shape
    t.original_bits = 8
    t.scale_block = 0
    t.scales_f16 = None
    t.dev = None
    return t


PHI3_MINI = dict(vocab_size=32064, hidden_size=3072, intermediate_size=8192, num_layers=32, num_heads=32,
                 num_kv_heads=32, head_dim=96, draft_layers=4, medusa_heads=0, max_seq_len=1024,
                 rope_theta=10000.0, norm_eps=1e-5)


def model_config(**kw) -> ModelConfig:
    c = ModelConfig()
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def tp_unique_id(lib: "Lib") -> bytes:
    """128-byte NCCL id for fl_engine_create_tp (make on one rank, share)."""
    b = np.zeros(128, np.uint8)
    lib.check(lib.fl_tp_unique_id(ptr(b)), "tp_unique_id")
    return b.tobytes()


def tp_layout(lib: "Lib", cfg: dict, rank: int, size: int) -> dict:
    out = np.zeros(9, np.int32)
    c = model_config(**cfg)
    lib.check(lib.fl_tp_layout(C.byref(c), rank, size, ptr(out)), "tp_layout")
    return dict(zip(("q0", "nq", "kv0", "nkv", "f0", "nf", "v0", "nv", "group"), (int(v) for v in out)))


class Engine:
    """Owns an fl_engine_t."""

    def __init__(self, lib: Lib, cfg: dict, device: int = 0, tp: tuple | None = None):
        """tp = (rank, size, nccl_id bytes from tp_unique_id) for a
        tensor-parallel rank; every rank then passes whole tensors."""
        self.lib = lib
        self.cfg = dict(cfg)
        self._c = model_config(**cfg)
        if tp is None:
            h = lib.fl_engine_create(C.byref(self._c), device)
        else:
            rank, size, uid = tp
            idb = np.frombuffer(bytes(uid), np.uint8).copy()
            h = lib.fl_engine_create_tp(C.byref(self._c), device, rank, size, ptr(idb))
        if not h:
            raise FLError(f"fl_engine_create failed: {lib.err()}")
        self.h = h

    def close(self):
        if self.h:
            self.lib.fl_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_linear(self, stack, layer, proj, w, d):
        self.lib.check(self.lib.fl_engine_load_linear(self.h, stack, layer, proj, ptr(w), ptr(d), w.shape[0],
                                                      w.shape[1]), "load_linear")

    def load_embedding(self, e):
        self.lib.check(self.lib.fl_engine_load_embedding(self.h, ptr(e)), "load_embedding")

    def set_weight_bits(self, bits):
        """4: the GEMV passes stream a packed 4-bit copy; 8: INT8 only."""
        self.lib.check(self.lib.fl_engine_set_weight_bits(self.h, bits), "set_weight_bits")

    def synthesize(self, seed):
        self.lib.check(self.lib.fl_engine_synthesize(self.h, seed), "synthesize")

    def forward_rows(self, stack, x, base, pos, mask=None, logits=True):
        x = np.ascontiguousarray(x, np.float32)
        M = x.shape[0]
        pos = np.ascontiguousarray(pos, np.int32)
        xo = np.empty_like(x)
        lg = np.empty((M, self.cfg["vocab_size"]), np.float32) if logits else None
        mk = None if mask is None else np.ascontiguousarray(mask, np.uint8)
        self.lib.check(self.lib.fl_engine_forward_rows(self.h, stack, ptr(x), M, base, ptr(pos), ptr(mk), ptr(xo),
                                                       ptr(lg)), "forward_rows")
        return xo, lg

    def greedy(self, prompt, n_new):
        p = np.ascontiguousarray(prompt, np.int32)
        o = np.empty(n_new, np.int32)
        self.lib.check(self.lib.fl_engine_greedy_generate(self.h, ptr(p), len(p), n_new, ptr(o)), "greedy")
        return o

    def spec_prefill(self, prompt, k, max_acc=-1):
        p = np.ascontiguousarray(prompt, np.int32)
        self.lib.check(self.lib.fl_engine_spec_prefill(self.h, ptr(p), len(p), k, max_acc), "spec_prefill")

    def spec_decode(self, n_new):
        o = np.empty(n_new, np.int32)
        acc = np.zeros(n_new + 1, np.int32)
        steps = C.c_int(0)
        self.lib.check(self.lib.fl_engine_spec_decode(self.h, n_new, ptr(o), ptr(acc), C.byref(steps)),
                       "spec_decode")
        return o, acc[: steps.value]

    def spec_generate(self, prompt, n_new, k, max_acc=-1):
        self.spec_prefill(prompt, k, max_acc)
        return self.spec_decode(n_new)

    def spec_generate_batch(self, prompts, n_new, k, seq_ids=None):
        """Decodes independent sequences (rows of `prompts`) together on this
        GPU (in-GPU batches as large as rows and memory allow) under the
        current rule; returns (tokens [nseq, n_new], steps [nseq], device
        seconds of the whole call, prefills included)."""
        pr = np.ascontiguousarray(prompts, np.int32)
        nseq, P = pr.shape
        ids = None if seq_ids is None else np.ascontiguousarray(seq_ids, np.uint32)
        out = np.empty((nseq, n_new), np.int32)
        steps = np.empty(nseq, np.int32)
        rc = self.lib.fl_engine_spec_generate_batch(self.h, ptr(pr), P, nseq, ptr(ids), n_new, k, ptr(out), ptr(steps))
        if rc < 0:
            self.lib.check(rc, "spec_generate_batch")
        return out, steps, self.last_timing()[2] * 1e-6

    def batch_reserve(self, nseq, max_ctx):
        """KV regions and buffers for an in-GPU batch of nseq sequences of up
        to max_ctx positions each."""
        self.lib.check(self.lib.fl_engine_batch_reserve(self.h, nseq, max_ctx), "batch_reserve")

    def batch_capacity(self):
        n, s = C.c_int(), C.c_int()
        self.lib.check(self.lib.fl_engine_batch_capacity(self.h, C.byref(n), C.byref(s)), "batch_capacity")
        return n.value, s.value

    def batch_prefill(self, prompts, k, seq_ids=None):
        pr = np.ascontiguousarray(prompts, np.int32)
        nseq, P = pr.shape
        ids = None if seq_ids is None else np.ascontiguousarray(seq_ids, np.uint32)
        self.lib.check(self.lib.fl_engine_batch_prefill(self.h, ptr(pr), P, nseq, ptr(ids), k), "batch_prefill")
        self._bn = nseq

    def batch_decode(self, n_new):
        """Decodes the prefilled batch: (tokens [nseq, n_new], steps [nseq],
        device seconds)."""
        out = np.empty((self._bn, n_new), np.int32)
        steps = np.empty(self._bn, np.int32)
        rc = self.lib.fl_engine_batch_decode(self.h, n_new, ptr(out), ptr(steps))
        if rc < 0:
            self.lib.check(rc, "batch_decode")
        return out, steps, self.last_timing()[2] * 1e-6

    def batch_begin(self, n_new):
        self.lib.check(self.lib.fl_engine_batch_begin(self.h, n_new), "batch_begin")

    def batch_step(self):
        """One step of every sequence: list of dict(n, produced, steps, accepted, done)."""
        s = np.zeros((self._bn, 5), np.int32)
        self.lib.check(self.lib.fl_engine_batch_step(self.h, ptr(s)), "batch_step")
        return [dict(zip(("n", "produced", "steps", "accepted", "done"), (int(v) for v in r))) for r in s]

    def batch_trace(self, seq):
        """sample_trace() of sequence `seq` of a sampled batch."""
        V = self.cfg["vocab_size"]
        t = dict(logits=np.empty((16, V), np.float32), qd=np.empty((7, V), np.uint32), qm=np.empty(7, np.uint64),
                 pt=np.empty((8, V), np.uint32), pm=np.empty(8, np.uint64), drafted=np.empty(7, np.int32))
        self.lib.check(self.lib.fl_engine_batch_trace(self.h, int(seq), ptr(t["logits"]), ptr(t["qd"]), ptr(t["qm"]),
                                                      ptr(t["pt"]), ptr(t["pm"]), ptr(t["drafted"])),
                       "batch_trace")
        return t

    def set_sampling(self, temperature, top_p=1.0, seed=0, seq_id=0):
        """temperature <= 0: greedy; > 0: Philox-keyed rejection sampling
        over top-p nucleus distributions (next spec_prefill onwards)."""
        self.lib.check(self.lib.fl_engine_set_sampling(self.h, float(temperature), float(top_p), int(seed) & 0xFFFFFFFF,
                                                       int(seq_id) & 0xFFFFFFFF), "set_sampling")

    def sample_trace_enable(self, on=True):
        self.lib.check(self.lib.fl_engine_sample_trace_enable(self.h, 1 if on else 0), "sample_trace_enable")

    def sample_trace(self):
        """dict(logits [16, V], qd [7, V] uint32, qm [7], pt [8, V] uint32,
        pm [8], drafted [7]) of the last step."""
        V = self.cfg["vocab_size"]
        t = dict(logits=np.empty((16, V), np.float32), qd=np.empty((7, V), np.uint32), qm=np.empty(7, np.uint64),
                 pt=np.empty((8, V), np.uint32), pm=np.empty(8, np.uint64), drafted=np.empty(7, np.int32))
        self.lib.check(self.lib.fl_engine_sample_trace(self.h, ptr(t["logits"]), ptr(t["qd"]), ptr(t["qm"]),
                                                       ptr(t["pt"]), ptr(t["pm"]), ptr(t["drafted"])),
                       "sample_trace")
        return t

    def spec_begin(self, n_new):
        self.lib.check(self.lib.fl_engine_spec_begin(self.h, n_new), "spec_begin")

    def spec_step(self):
        """One speculative step: dict(n, produced, steps, accepted, done)."""
        s = np.zeros(5, np.int32)
        self.lib.check(self.lib.fl_engine_spec_step(self.h, ptr(s)), "spec_step")
        return dict(zip(("n", "produced", "steps", "accepted", "done"), (int(v) for v in s)))

    def get_sampling(self):
        t, p, s, q = C.c_float(), C.c_float(), C.c_uint32(), C.c_uint32()
        self.lib.check(self.lib.fl_engine_get_sampling(self.h, C.byref(t), C.byref(p), C.byref(s), C.byref(q)),
                       "get_sampling")
        return t.value, p.value, s.value, q.value

    def last_timing(self):
        a, b, c = C.c_double(), C.c_double(), C.c_double()
        self.lib.check(self.lib.fl_engine_last_timing(self.h, C.byref(a), C.byref(b), C.byref(c)), "timing")
        return a.value, b.value, c.value

    def stream(self) -> int:
        return self.lib.fl_engine_stream(self.h)

    def last_launches(self) -> int:
        return self.lib.fl_engine_last_launches(self.h)

    def step_kernel(self) -> bool:
        """True when the current step graph is the one-kernel step."""
        return bool(self.lib.fl_engine_step_kernel(self.h))

    def step_trace(self, cap=4096):
        """(t [n,6] uint64 ns, desc [n,4] int32) of the last step-kernel
        launch; empty when FL_STEP_TRACE=1 was not set at graph build."""
        t = np.zeros((cap, 6), np.uint64)
        d = np.zeros((cap, 4), np.int32)
        n = self.lib.fl_engine_step_trace(self.h, ptr(t), ptr(d), cap)
        if n < 0:
            self.lib.check(n, "step_trace")
        return t[:n], d[:n]

    def medusa_generate(self, prompt, n_new, topk, max_nodes):
        """Medusa greedy decoding: (tokens, accepted count per step)."""
        p = np.ascontiguousarray(prompt, np.int32)
        tk = np.ascontiguousarray(topk, np.int32)
        o = np.empty(n_new, np.int32)
        acc = np.zeros(n_new + 1, np.int32)
        steps = C.c_int(0)
        self.lib.check(self.lib.fl_engine_medusa_generate(self.h, ptr(p), len(p), n_new, ptr(tk), len(tk), max_nodes,
                                                          ptr(o), ptr(acc), C.byref(steps)), "medusa_generate")
        return o, acc[: steps.value]

    def spec_medusa_generate(self, prompt, n_new, k, topk, max_nodes):
        """Draft chain + Medusa tree, greedy: (tokens, accepted count per step)."""
        p = np.ascontiguousarray(prompt, np.int32)
        tk = np.ascontiguousarray(topk, np.int32)
        o = np.empty(n_new, np.int32)
        acc = np.zeros(n_new + 1, np.int32)
        steps = C.c_int(0)
        self.lib.check(self.lib.fl_engine_spec_medusa_generate(self.h, ptr(p), len(p), n_new, k, ptr(tk), len(tk),
                                                               max_nodes, ptr(o), ptr(acc), C.byref(steps)),
                       "spec_medusa_generate")
        return o, acc[: steps.value]

    def spec_tree_generate(self, prompt, n_new, k, width):
        """Static draft tree (chain + top-width per depth), greedy:
        (tokens, accepted count per step)."""
        p = np.ascontiguousarray(prompt, np.int32)
        o = np.empty(n_new, np.int32)
        acc = np.zeros(n_new + 1, np.int32)
        steps = C.c_int(0)
        self.lib.check(self.lib.fl_engine_spec_tree_generate(self.h, ptr(p), len(p), n_new, k, width, ptr(o), ptr(acc),
                                                             C.byref(steps)), "spec_tree_generate")
        return o, acc[: steps.value]

    def batch_tree_generate(self, prompts, n_new, k, width):
        """Static draft tree for an in-GPU batch (after batch_reserve):
        (tokens [nseq, n_new], steps [nseq], device seconds of the decode)."""
        pr = np.ascontiguousarray(prompts, np.int32)
        nseq, P = pr.shape
        out = np.empty((nseq, n_new), np.int32)
        steps = np.empty(nseq, np.int32)
        rc = self.lib.fl_engine_batch_tree_generate(self.h, ptr(pr), P, nseq, n_new, k, width, ptr(out), ptr(steps))
        if rc < 0:
            self.lib.check(rc, "batch_tree_generate")
        return out, steps, self.last_timing()[2] * 1e-6

    def step_trace_stages(self):
        """[64, 4] uint64 stage stamps of the phase FL_STEP_TRACE_PHASE names."""
        t = np.zeros((64, 8), np.uint64)
        self.lib.fl_engine_step_trace_stages(self.h, ptr(t))
        return t

    def bench_attention(self, stack, M, ctx, reps=10):
        us = C.c_double()
        self.lib.check(self.lib.fl_engine_bench_attention(self.h, stack, M, ctx, reps, C.byref(us)),
                       "bench_attention")
        return us.value

    def bench_linear(self, stack, kind, M, reps=10):
        us, by = C.c_double(), C.c_double()
        self.lib.check(self.lib.fl_engine_bench_linear(self.h, stack, kind, M, reps, C.byref(us), C.byref(by)),
                       "bench_linear")
        return us.value, by.value
