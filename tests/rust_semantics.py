"""Independent pure-Python (numpy float32) restatement of selected Rust
semantics of the reference, used to cross-check the C++ host library on
small random inputs.  Deliberately written in a different style (scalar
numpy float32 arithmetic) from csrc/host."""
import struct

import numpy as np

F32 = np.float32
Q = F32(8388608.0)
M64 = (1 << 64) - 1


def from_f32(x):
    out = []
    for v in np.asarray(x, dtype=np.float32):
        s = F32(v) * Q
        if s >= F32(2147483648.0):
            out.append(2**31 - 1)
        elif s <= F32(-2147483648.0):
            out.append(-(2**31))
        elif np.isnan(s):
            out.append(0)
        else:
            a = abs(float(s))
            r = np.floor(a + 0.5) if a - np.floor(a) != 0.5 else np.floor(a) + 1.0
            out.append(int(r) if s >= 0 else -int(r))
    return np.asarray(out, dtype=np.int32)


def to_f32(q):
    return np.asarray([F32(F32(int(v)) / Q) for v in q], dtype=np.float32)


def fmix64(h):
    h ^= h >> 33
    h = (h * 0xFF51AFD7ED558CCD) & M64
    h ^= h >> 33
    h = (h * 0xC4CEB9FE1A85EC53) & M64
    h ^= h >> 33
    return h


def stochastic_int4(q, seed, counter):
    f = to_f32(q)
    if f.size == 0:
        return b"", 1.0, counter
    mx = F32(0.0)
    for v in f:
        mx = max(mx, abs(v))
    scale = F32(mx / F32(7.5)) if mx > F32(1e-9) else F32(1.0)
    out = bytearray()
    for i in range(0, f.size, 2):
        byte = 0
        for j in range(2):
            if i + j >= f.size:
                break
            v = F32(f[i + j] / scale)
            fl = F32(np.floor(v))
            frac = F32(v - fl)
            h = fmix64((seed ^ counter) & M64)
            counter += 1
            r = F32(np.uint64(h).astype(np.float32) / F32(18446744073709551616.0))  # one rounding, as Rust's `as f32`
            qq = int(fl) + 1 if r < frac else int(fl)
            qq = min(max(qq, -8), 7)
            nib = qq & 0xF
            byte |= (nib << 4) if j == 0 else nib
        out.append(byte)
    return bytes(out), float(scale), counter


def eb_quantize(q, eps):
    scale = F32(2.0) * F32(eps)
    out = bytearray()
    for v in to_f32(q):
        r = np.round(F32(v / scale))  # numpy rounds half to even -> fix below
        x = float(F32(v / scale))
        r = np.floor(abs(x) + 0.5) * (1 if x >= 0 else -1) if abs(x) - np.floor(abs(x)) == 0.5 else np.round(x)
        r = min(max(r, -32768.0), 32767.0)
        out += struct.pack("<h", int(r))
    return bytes(out), float(scale)


def block_sparse(q, eps):
    scale = F32(2.0) * F32(eps)
    codes = np.frombuffer(eb_quantize(q, eps)[0], dtype="<i2")
    n = codes.size
    out = bytearray(struct.pack("<I", n))
    for b in range(0, n, 32):
        blk = codes[b:b + 32]
        mask = 0
        vals = bytearray()
        for i, c in enumerate(blk):
            if c != 0:
                mask |= 1 << i
                vals += struct.pack("<h", int(c))
        out += struct.pack("<I", mask) + vals
    return bytes(out), float(scale)
