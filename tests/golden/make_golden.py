"""Generates tests/golden/kat_blocks.json -- known-answer GGML blocks.

The reference (llama.rs) ships no golden vectors and cannot be built in this
image, so these known answers come from a second, independent restatement of
its decoders written here in plain Python with numpy float32 scalars
(value_at, src/quant.rs:349-456; dot_row_scalar, src/quant.rs:458-648).  The
blocks are deterministic byte patterns -- the same construction the
reference's own Q5_K test uses (src/quant.rs:1016-1023: byte i =
i*73 + 19 mod 256) -- with the f16 scale fields overwritten by fixed finite
values.  The C oracle and the CUDA kernels must reproduce every dequantized
value bit for bit.

Run:  python tests/golden/make_golden.py
"""
import json
import math
import os

import numpy as np

F = np.float32
TYPES = {  # ggml id: (name, block values, block bytes, f16 fields (offset, value))
    0: ("F32", 1, 4, []),
    1: ("F16", 1, 2, []),
    30: ("BF16", 1, 2, []),
    2: ("Q4_0", 32, 18, [(0, 0.0123)]),
    3: ("Q4_1", 32, 20, [(0, 0.0071), (2, -0.051)]),
    6: ("Q5_0", 32, 22, [(0, 0.0044)]),
    7: ("Q5_1", 32, 24, [(0, 0.0029), (2, -0.047)]),
    8: ("Q8_0", 32, 34, [(0, 0.00081)]),
    12: ("Q4_K", 256, 144, [(0, 0.003), (2, 0.001)]),
    13: ("Q5_K", 256, 176, [(0, 0.003), (2, 0.001)]),
    14: ("Q6_K", 256, 210, [(208, 0.00042)]),
}


def f16(b, o):
    return F(np.frombuffer(bytes(b[o:o + 2]), dtype=np.float16)[0])


def bf16(b, o):
    return F(np.frombuffer(bytes([0, 0, b[o], b[o + 1]]), dtype="<f4")[0])


def scale_min_k4(i, s):
    if i < 4:
        return s[i] & 63, s[i + 4] & 63
    return (s[i + 4] & 0x0F) | ((s[i - 4] >> 6) << 4), (s[i + 4] >> 4) | ((s[i] >> 6) << 4)


def value_at(row, t, col):
    if t == 0:
        return F(np.frombuffer(bytes(row[col * 4:col * 4 + 4]), dtype="<f4")[0])
    if t == 1:
        return f16(row, col * 2)
    if t == 30:
        return bf16(row, col * 2)
    if t in (2, 3):
        bs, qo = (18, 2) if t == 2 else (20, 4)
        b = row[col // 32 * bs:][:bs]
        j = col % 32
        q = b[qo + j] & 15 if j < 16 else b[qo + j - 16] >> 4
        if t == 2:
            return f16(b, 0) * (F(q) - F(8))
        return f16(b, 0) * F(q) + f16(b, 2)
    if t in (6, 7):
        bs = 22 if t == 6 else 24
        qh_off, qs_off = (2, 6) if t == 6 else (4, 8)
        b = row[col // 32 * bs:][:bs]
        j = col % 32
        low = b[qs_off + j] & 15 if j < 16 else b[qs_off + j - 16] >> 4
        high = (b[qh_off + j // 8] >> (j % 8)) & 1
        q = low | (high << 4)
        if t == 6:
            return f16(b, 0) * (F(q) - F(16))
        return f16(b, 0) * F(q) + f16(b, 2)
    if t == 8:
        b = row[col // 32 * 34:][:34]
        return f16(b, 0) * F(np.int8(np.uint8(b[2 + col % 32])))
    if t == 12:
        b = row[col // 256 * 144:][:144]
        j = col % 256
        g = j // 32
        sc, mn = scale_min_k4(g, b[4:16])
        packed = b[16 + (g // 2) * 32 + j % 32]
        q = packed & 15 if g % 2 == 0 else packed >> 4
        return f16(b, 0) * F(sc) * F(q) - f16(b, 2) * F(mn)
    if t == 13:
        b = row[col // 256 * 176:][:176]
        j = col % 256
        g = j // 32
        sc, mn = scale_min_k4(g, b[4:16])
        packed = b[48 + g // 2 * 32 + j % 32]
        low = packed & 15 if g % 2 == 0 else packed >> 4
        high = 16 if b[16 + j % 32] & (1 << g) else 0
        return f16(b, 0) * F(sc) * F(low + high) - f16(b, 2) * F(mn)
    if t == 14:
        b = row[col // 256 * 210:][:210]
        j = col % 256
        half, within = j // 128, j % 128
        lane, quarter = within % 32, within // 32
        ql = [b[half * 64 + lane] & 15, b[half * 64 + 32 + lane] & 15,
              b[half * 64 + lane] >> 4, b[half * 64 + 32 + lane] >> 4][quarter]
        qh = (b[128 + half * 32 + lane] >> (quarter * 2)) & 3
        q = F((ql | (qh << 4)) - 32)
        scale = F(np.int8(np.uint8(b[192 + half * 8 + quarter * 2 + lane // 16])))
        return f16(b, 208) * scale * q
    raise ValueError(t)


def dot_order(t, cols):
    """Column order in which dot_row_scalar accumulates (src/quant.rs:458-648)."""
    if t in (2, 3, 6, 7):
        return [bi * 32 + j + h for bi in range(cols // 32) for j in range(16) for h in (0, 16)]
    if t == 14:
        return [bi * 256 + half * 128 + k * 32 + lane for bi in range(cols // 256)
                for half in range(2) for lane in range(32) for k in range(4)]
    return list(range(cols))


def dot_row_scalar(row, t, x, cols):
    # Every per-type product in dot_row_scalar equals value_at(col) * x[col]
    # (same f32 operations in the same order), summed in dot_order.
    s = F(0)
    for c in dot_order(t, cols):
        s = F(s + value_at(row, t, c) * F(x[c]))
    return s


def make_rows(t, nrows):
    name, bv, bb, fields = TYPES[t]
    cols = 64 if bv != 256 else 256
    rb = cols // bv * bb
    data = bytearray(((i * 73 + 19 + 31 * t) & 0xFF) for i in range(nrows * rb))
    if t == 0:
        vals = np.array([math.sin(i * 0.37) * 0.7 for i in range(nrows * cols)], dtype="<f4")
        data = bytearray(vals.tobytes())
    elif t == 1:
        vals = np.array([math.cos(i * 0.29) * 3.0 for i in range(nrows * cols)], dtype="<f2")
        data = bytearray(vals.tobytes())
    elif t == 30:
        vals = np.array([math.sin(i * 0.11) * 5.0 for i in range(nrows * cols)], dtype="<f4")
        data = bytearray((vals.view("<u4") >> 16).astype("<u2").tobytes())
    else:
        for r in range(nrows):
            for blk in range(cols // bv):
                base = r * rb + blk * bb
                for off, v in fields:
                    h = np.array([v * (1 + 0.25 * blk + 0.5 * r)], dtype="<f2").tobytes()
                    data[base + off:base + off + 2] = h
    return cols, rb, bytes(data)


def main():
    out = {"note": __doc__.strip().splitlines()[0], "cases": []}
    x_all = [math.sin(i * 0.037) for i in range(256)]  # the input of src/quant.rs:1007
    for t in TYPES:
        nrows = 2
        cols, rb, data = make_rows(t, nrows)
        x = np.array(x_all[:cols], dtype=np.float32)
        vals, dots = [], []
        for r in range(nrows):
            row = data[r * rb:(r + 1) * rb]
            vals.append([int(np.float32(value_at(row, t, c)).view(np.uint32)) for c in range(cols)])
            dots.append(int(np.float32(dot_row_scalar(row, t, x, cols)).view(np.uint32)))
        out["cases"].append(dict(type=t, name=TYPES[t][0], rows=nrows, cols=cols,
                                 data=data.hex(), value_bits=vals, dot_bits=dots))
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat_blocks.json")
    with open(path, "w") as f:
        json.dump(out, f)
    print("wrote", path)


if __name__ == "__main__":
    main()
