"""Seeded small models shared by the CPU and GPU tests."""
import numpy as np

# d, ffn and q_dim multiples of 512 take the TMA-ring GEMV; SMALL_V1 (d 256)
# takes the register-streamed fallback kernel.
SMALL = dict(vocab=1000, d=512, ffn=1024, layers=2, heads=8, kv_heads=8, head_dim=64, theta=10000.0, eps=1e-5)
SMALL_GQA = dict(SMALL, kv_heads=4)
SMALL_V1 = dict(vocab=512, d=256, ffn=512, layers=2, heads=4, kv_heads=4, head_dim=64, theta=10000.0, eps=1e-5)


def engine_cfg(dims, draft_layers=1, medusa_heads=0, max_seq_len=256):
    return dict(vocab_size=dims["vocab"], hidden_size=dims["d"], intermediate_size=dims["ffn"],
                num_layers=dims["layers"], num_heads=dims["heads"], num_kv_heads=dims["kv_heads"],
                head_dim=dims["head_dim"], draft_layers=draft_layers, medusa_heads=medusa_heads,
                max_seq_len=max_seq_len, rope_theta=dims["theta"], norm_eps=dims["eps"])


def make_weights(lib, dims, seed, draft_layers=1, medusa_heads=0, std=0.02):
    """(stack, layer, proj) -> (int8, fp16 bits) from the seeded Q4_0 generator,
    plus the f32 embedding table."""
    from flb200 import tensor_id
    d, F, qd, kd = dims["d"], dims["ffn"], dims["heads"] * dims["head_dim"], dims["kv_heads"] * dims["head_dim"]
    shapes = [(qd, d), (kd, d), (kd, d), (d, qd), (F, d), (F, d), (d, F)]
    w = {}
    for s, nl in ((0, dims["layers"]), (1, draft_layers)):
        for l in range(nl):
            for p, (r, c) in enumerate(shapes):
                w[(s, l, p)] = lib.synth_q4_0_i8(seed, tensor_id(s, l, p), r, c, std)
    for h in range(medusa_heads):
        w[(2, h, 0)] = lib.synth_q4_0_i8(seed, tensor_id(2, h, 0), d, d, std)
    w[(3, 0, 1)] = lib.synth_q4_0_i8(seed, tensor_id(3, 0, 1), dims["vocab"], d, std)
    embed = lib.synth_q4_0_f32(seed, tensor_id(3, 0, 0), dims["vocab"], d, std)
    return w, embed


def load_engine(eng, w, embed):
    for (s, l, p), (wq, dq) in w.items():
        eng.load_linear(s, l, p, wq, dq)
    eng.load_embedding(embed)


def prompt(seed, n, vocab):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)
