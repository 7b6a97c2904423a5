"""Tensor parallelism: the shard layout (CPU) and a 2-rank decode on two GPUs
(skipped with fewer) that must give identical streams on both ranks, equal
to the oracle's under the near-tie rule."""
import ctypes as C

import numpy as np
import pytest

import flb200

PHI3_MEDIUM = dict(vocab_size=32064, hidden_size=5120, intermediate_size=17920, num_layers=40, num_heads=40,
                   num_kv_heads=10, head_dim=128, draft_layers=2, medusa_heads=0, max_seq_len=4096,
                   rope_theta=10000.0, norm_eps=1e-5)


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_layout_covers_the_model(lib, size):
    L = [flb200.tp_layout(lib, PHI3_MEDIUM, r, size) for r in range(size)]
    H, Hkv, F, V = 40, 10, 17920, 32064
    G = H // Hkv
    assert sum(l["nq"] for l in L) == H and [l["q0"] for l in L] == [r * H // size for r in range(size)]
    assert sum(l["nf"] for l in L) == F and sum(l["nv"] for l in L) == V
    for l in L:
        assert l["group"] == G and l["nf"] % 32 == 0 and (l["q0"] * 128) % 32 == 0
        needed = {q // G for q in range(l["q0"], l["q0"] + l["nq"])}
        assert needed == set(range(l["kv0"], l["kv0"] + l["nkv"]))
    # straddling KV heads are held by both neighbours at 4 and 8 ranks
    held = sum(l["nkv"] for l in L)
    assert held == Hkv if size <= 2 else held > Hkv


def test_layout_rejects_bad_splits(lib):
    bad = dict(PHI3_MEDIUM, num_heads=12, num_kv_heads=4)
    with pytest.raises(flb200.FLError):
        flb200.tp_layout(lib, bad, 0, 8)


TP_GQA = dict(vocab=1024, d=512, ffn=1024, layers=2, heads=12, kv_heads=3, head_dim=64, theta=10000.0, eps=1e-5)


def _rank(rank, size, uid, q, fused="0"):
    import sys, os
    os.environ["FL_TP_FUSED"] = fused
    sys.path[:0] = [os.path.dirname(__file__), os.path.join(os.path.dirname(__file__), "..", "fast-llm-inference_b200")]
    import flb200 as F
    from _model import engine_cfg, load_engine, make_weights, prompt
    try:
        lib = F.Lib()
        lib.check(lib.fl_cuda_init(rank), "init")
        w, embed = make_weights(lib, TP_GQA, seed=41)
        eng = F.Engine(lib, engine_cfg(TP_GQA, draft_layers=1), rank, tp=(rank, size, uid))
        load_engine(eng, w, embed)
        p = prompt(8, 16, TP_GQA["vocab"])
        toks, acc = eng.spec_generate(p, 24, 4)
        g = eng.greedy(p, 12)
        # three sequences as one in-GPU batch (15 verify rows: NCCL sums;
        # 3-row draft passes: the fused NVLink push)
        eng.batch_reserve(3, 12 + 24 + 4 + 3)
        eng.batch_prefill(_batch_prompts(prompt), 4)
        bt, _, _ = eng.batch_decode(24)
        # a 17-node draft tree (k = 4, width 4): merged top-4 across the ranks
        tt, _ = eng.spec_tree_generate(p, 24, 4, 4)
        # the same tree for each sequence of a batch of three
        eng.batch_reserve(3, 12 + 24 + 1 + 4 * 4 + 4 + 3)
        btt, _, _ = eng.batch_tree_generate(_batch_prompts(prompt), 24, 4, 4)
        eng.close()
        q.put((rank, toks.tolist(), acc.tolist(), g.tolist(), bt.tolist(), tt.tolist(), btt.tolist(), None))
    except Exception as ex:  # reported to the parent
        q.put((rank, None, None, None, None, None, None, repr(ex)))


def _batch_prompts(prompt):
    return np.stack([prompt(70 + i, 12, TP_GQA["vocab"]) for i in range(3)])


@pytest.mark.gpu
@pytest.mark.parametrize("fused", ["0", "1"])
def test_two_rank_decode_matches_oracle(gpu, orc, fused):
    """Two tensor-parallel ranks (one process per GPU) against the oracle,
    with the decode-sized all-reduces on NCCL (the default) or on the fused
    NVLink push (FL_TP_FUSED=1)."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from _model import make_weights, prompt
    import bind
    uid = flb200.tp_unique_id(gpu)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, q, fused)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, toks, acc, g, bt, tt, btt, err = q.get(timeout=600)
        assert err is None, f"rank {r}: {err}"
        res[r] = (np.array(toks), np.array(acc), np.array(g), np.array(bt), np.array(tt), np.array(btt))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][2], res[1][2]), "ranks disagree"
    assert np.array_equal(res[0][3], res[1][3]), "ranks disagree on the batch"
    assert np.array_equal(res[0][4], res[1][4]), "ranks disagree on the tree decode"
    assert np.array_equal(res[0][5], res[1][5]), "ranks disagree on the batched tree decode"
    w, embed = make_weights(gpu, TP_GQA, seed=41)
    om = bind.OracleModel(orc, TP_GQA, embed, w, draft_layers=1)
    p = prompt(8, 16, TP_GQA["vocab"])
    want, _, margins = om.spec(p, 24, 4)
    td = np.nonzero(res[0][4] != want)[0]
    assert td.size == 0 or margins[td[0]] < 1e-2, f"tree decode diverges at {td[:1]}"
    got = res[0][0]
    diff = np.nonzero(got != want)[0]
    assert diff.size == 0 or margins[diff[0]] < 1e-2, f"diverges at {diff[:1]} (margin {margins[diff[0]]:.3g})"
    gw, gm = om.greedy(p, 12)
    gd = np.nonzero(res[0][2] != gw)[0]
    assert gd.size == 0 or gm[gd[0]] < 1e-2
    for i, pb in enumerate(_batch_prompts(prompt)):
        bw, bm = om.greedy(pb, 24)
        bd = np.nonzero(res[0][3][i] != bw)[0]
        assert bd.size == 0 or bm[bd[0]] < 1e-2, f"batch sequence {i} diverges at {bd[:1]}"
        td = np.nonzero(res[0][5][i] != bw)[0]
        assert td.size == 0 or bm[td[0]] < 1e-2, f"batched tree sequence {i} diverges at {td[:1]}"


@pytest.mark.gpu
def test_bounded_wait_reports_timeout(gpu):
    """A device wait that runs out (arrival counters nobody increments)
    ends the kernel, sets the error word, and fl_cuda_sync reports
    FL_E_TIMEOUT once; the device stays usable afterwards."""
    import time
    FL_E_TIMEOUT = -5
    t0 = time.time()
    assert gpu.fl_cuda_tp_wait_timeout_check() == 0, gpu.err()
    assert time.time() - t0 < 30
    assert gpu.fl_cuda_sync() == FL_E_TIMEOUT
    assert gpu.fl_cuda_sync() == 0
    w, d = gpu.synth_q4_0_i8(3, 77, 64, 256)
    from test_gemv_gpu import Dev
    import ctypes as C
    from flb200 import block_tensor
    t = block_tensor(w, d)
    assert gpu.fl_cuda_upload_tensor(C.byref(t)) == 0
    A = np.ones((1, 256), np.float32)
    dA = Dev(gpu, A.nbytes).put(A)
    dO = Dev(gpu, 64 * 4)
    assert gpu.fl_cuda_matmul_i8(dA.p, C.byref(t), dO.p, 1, 64, 256, None) == 0
    assert gpu.fl_cuda_sync() == 0


# ---------------------------------------------------------------------------
# The tensor-parallel control flow on CPU (gloo, world size 2): every rank
# holds its vocabulary slice of the LM-head logits (fl_tp_layout), forms its
# local best keys (fl_argmax_key, global indices), the keys are all-gathered,
# and the argmax (largest key) and the draft-tree candidates
# (fl_tp_merge_topw) must equal those of the whole row on every rank.
# ---------------------------------------------------------------------------

def _tp_worker(rank, world, port, q):
    import os
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = flb200.Lib()
        cfg = dict(vocab_size=1001, hidden_size=512, intermediate_size=1024, num_layers=2, num_heads=8,
                   num_kv_heads=4, head_dim=64, draft_layers=1, medusa_heads=0, max_seq_len=64, rope_theta=1e4,
                   norm_eps=1e-5)
        lay = flb200.tp_layout(lib, cfg, rank, world)
        v0, nv = lay["v0"], lay["nv"]
        rows, width = 6, 8
        rng = np.random.default_rng(99)
        logits = rng.standard_normal((rows, 1001)).astype(np.float32)
        logits[2, 17] = logits[2, 900] = logits[2].max() + 1.0  # a tie across the two slices
        local = logits[:, v0:v0 + nv]
        keys = np.zeros((rows, width), np.uint64)
        for r in range(rows):
            k = np.array([lib.fl_argmax_key(float(v), v0 + i) for i, v in enumerate(local[r])], np.uint64)
            keys[r] = np.sort(k)[::-1][:width]
        allk = [torch.zeros(rows * width, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allk, torch.from_numpy(keys.view(np.int64).reshape(-1)))
        gathered = np.stack([t.numpy().view(np.uint64).reshape(rows, width) for t in allk])  # [rank, row, w]
        best = [0x7fffffff - (int(gathered[:, r, 0].max()) & 0xffffffff) for r in range(rows)]
        top = []
        for r in range(rows):
            flat = np.ascontiguousarray(gathered[:, r, :].reshape(-1))
            tok = np.zeros(width, np.int32)
            assert lib.fl_tp_merge_topw(flat.ctypes.data_as(C.c_void_p), world, width, width,
                                        tok.ctypes.data_as(C.c_void_p)) == 0
            top.append(tok.tolist())
        q.put((rank, best, top))
    finally:
        dist.destroy_process_group()


def test_tp_argmax_and_candidates_merge_gloo():
    import multiprocessing
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = multiprocessing.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=60) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(99)
    logits = rng.standard_normal((6, 1001)).astype(np.float32)
    logits[2, 17] = logits[2, 900] = logits[2].max() + 1.0
    want_best = [int(np.argmax(r)) for r in logits]                    # first maximum wins
    want_top = [np.lexsort((np.arange(1001), -r))[:8].tolist() for r in logits]  # value desc, index asc
    for rank, best, top in res:
        assert best == want_best, rank
        assert top == want_top, rank
    assert want_best[2] == 17
