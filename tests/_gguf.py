"""A minimal GGUF v3 writer for tests: Q4_0 (18-byte blocks, fp16 d, low
nibbles = elements 0..15, high = 16..31) and F32 tensors, built from the
seeded generator's INT8 q-8 values and fp16 block scales."""
import struct

import numpy as np

Q4_0, F32 = 2, 0


def q4_0_bytes(w, d):
    """INT8 [-8, 7] [rows, cols] + fp16 bits [rows, cols/32] -> Q4_0 blocks."""
    rows, cols = w.shape
    q = (w.astype(np.int16) + 8).astype(np.uint8).reshape(rows, cols // 32, 32)
    qs = (q[:, :, :16] & 0xF) | ((q[:, :, 16:] & 0xF) << 4)
    blocks = np.zeros((rows, cols // 32, 18), np.uint8)
    blocks[:, :, :2] = d.astype(np.uint16).reshape(rows, cols // 32, 1).view(np.uint8)
    blocks[:, :, 2:] = qs
    return blocks.tobytes()


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, tensors, align=32):
    """tensors: list of (name, kind, payload) with kind "q4_0" (payload (w, d))
    or "f32" (payload [rows, cols] float32)."""
    infos, datas = [], []
    off = 0
    for name, kind, payload in tensors:
        if kind == "q4_0":
            w, d = payload
            data, typ, dims = q4_0_bytes(w, d), Q4_0, (w.shape[1], w.shape[0])
        else:
            a = np.ascontiguousarray(payload, np.float32)
            data, typ, dims = a.tobytes(), F32, (a.shape[1], a.shape[0])
        pad = (-off) % align
        off += pad
        datas.append(b"\0" * pad + data)
        infos.append(_str(name) + struct.pack("<I", 2) + struct.pack("<QQ", *dims) + struct.pack("<I", typ) +
                     struct.pack("<Q", off))
        off += len(data)
    kv = _str("general.architecture") + struct.pack("<I", 8) + _str("phi3")
    kv += _str("general.alignment") + struct.pack("<I", 4) + struct.pack("<I", align)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), 2) + kv + b"".join(infos)
    head += b"\0" * ((-len(head)) % align)
    with open(path, "wb") as f:
        f.write(head + b"".join(datas))
