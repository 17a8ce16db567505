"""Shared cases for the forward-pass ops (matmul formats, rmsnorm, silu,
ffn_swiglu, vec_add, sample_argmax): the reference suite's own known-answer
tests restated (src/test_ops.cpp, cited per case) and a float64 dequantiser
of the GGUF block layouts (src/gguf.h:54-135) for tolerance checks.

Each known-answer case is run against a `backend` object with the oracle's
method names (oracle.port(), oracle.reference(), or the GPU adapter in
test_forward_gpu.py)."""
import numpy as np

F32, F16, Q4_0, Q8_0, Q6_K = 0, 1, 2, 8, 14


def f16_bytes(vals):
    return np.asarray(vals, np.float16).view(np.uint8)


def q8_block(d_bits, qs):
    b = np.zeros(34, np.uint8)
    b[0:2] = np.array([d_bits], np.uint16).view(np.uint8)
    b[2:] = np.asarray(qs, np.int8).view(np.uint8)
    return b


def q4_block(d_bits, byte):
    b = np.zeros(18, np.uint8)
    b[0:2] = np.array([d_bits], np.uint16).view(np.uint8)
    b[2:] = byte
    return b


def q6_block(d_bits, qh_byte, scale=1):
    b = np.zeros(210, np.uint8)
    b[128:192] = qh_byte
    b[192:208] = np.full(16, scale, np.int8).view(np.uint8)
    b[208:210] = np.array([d_bits], np.uint16).view(np.uint8)
    return b


def matmul_kats():
    """(name, W bytes, x, rows, cols, type, expected, tol) from test_ops.cpp."""
    ones32 = np.ones(32, np.float32)
    cases = [
        ("f32 2x3 (test_ops.cpp:42-56)", np.array([1, 2, 3, 4, 5, 6], np.float32).view(np.uint8),
         np.ones(3, np.float32), 2, 3, F32, [6.0, 15.0], 1e-4),
        ("f32 identity (test_ops.cpp:58-68)", np.eye(4, dtype=np.float32).view(np.uint8).ravel(),
         np.array([3.14, 2.71, 1.41, 1.73], np.float32), 4, 4, F32, [3.14, 2.71, 1.41, 1.73], 1e-4),
        ("f16 2x2 (test_ops.cpp:71-89)",
         np.array([0x4000, 0x0000, 0x0000, 0x4200], np.uint16).view(np.uint8),
         np.array([5.0, 7.0], np.float32), 2, 2, F16, [10.0, 21.0], 1e-4),
        ("f32 256 identity (test_ops.cpp:548-576)",
         np.eye(256, dtype=np.float32).view(np.uint8).ravel(), np.arange(256, dtype=np.float32),
         256, 256, F32, list(range(256)), 1e-4),
        ("q8_0 d=1 qs=2 (test_ops.cpp:641-655)", q8_block(0x3C00, [2] * 32), ones32, 1, 32, Q8_0,
         [64.0], 0.1),
        ("q8_0 d=0.5 qs=0..31 (test_ops.cpp:658-671)", q8_block(0x3800, range(32)), ones32, 1, 32,
         Q8_0, [248.0], 0.5),
        ("q8_0 two rows (test_ops.cpp:674-695)",
         np.concatenate([q8_block(0x3C00, [1] * 32)] * 2 + [q8_block(0x4000, [1] * 32)] * 2),
         np.ones(64, np.float32), 2, 64, Q8_0, [64.0, 128.0], 0.5),
        ("q8_0 dispatch (test_ops.cpp:697-709)", q8_block(0x3C00, [3] * 32), ones32, 1, 32, Q8_0,
         [96.0], 0.5),
        ("q4_0 nibbles 9 (test_ops.cpp:717-734)", q4_block(0x3C00, 0x99), ones32, 1, 32, Q4_0,
         [32.0], 0.5),
        ("q4_0 nibbles 8 (test_ops.cpp:737-752)", q4_block(0x4000, 0x88), ones32, 1, 32, Q4_0,
         [0.0], 0.5),
        ("q4_0 dispatch (test_ops.cpp:755-769)", q4_block(0x3C00, 0xAA), ones32, 1, 32, Q4_0,
         [64.0], 0.5),
        ("q6_k q=-32 (test_ops.cpp:777-793)", q6_block(0x3C00, 0x00), np.ones(256, np.float32), 1,
         256, Q6_K, [-8192.0], 1.0),
        ("q6_k q=0 (test_ops.cpp:796-813)", q6_block(0x3C00, 0xAA), np.ones(256, np.float32), 1,
         256, Q6_K, [0.0], 1.0),
        ("q6_k two rows d=2 (test_ops.cpp:833-850)",
         np.concatenate([q6_block(0x4000, 0x00)] * 2), np.ones(256, np.float32), 2, 256, Q6_K,
         [-16384.0, -16384.0], 1.0),
        ("q8_0 8x64 d=0.5 (test_ops.cpp:856-899)",
         np.concatenate([q8_block(0x3800, [1] * 32)] * 16), np.ones(64, np.float32), 8, 64, Q8_0,
         [32.0] * 8, 0.5),
        ("f32 8x64 all 2 (test_ops.cpp:901-918)", np.full(8 * 64, 2.0, np.float32).view(np.uint8),
         np.ones(64, np.float32), 8, 64, F32, [128.0] * 8, 0.5),
    ]
    return cases


def silu_ref(v):
    v = np.float32(v)
    return v * (np.float32(1) / (np.float32(1) + np.exp(-v, dtype=np.float32)))


# ---------------------------------------------------------------- dequant
def _f16(u8):
    return u8.view(np.float16).astype(np.float64)


def dequant(W: np.ndarray, wtype: int, rows: int, cols: int) -> np.ndarray:
    """float64 [rows][cols] values of GGUF-layout weights."""
    if wtype == F32:
        return W.view(np.float32).reshape(rows, cols).astype(np.float64)
    if wtype == F16:
        return W.view(np.float16).reshape(rows, cols).astype(np.float64)
    if wtype == Q4_0:
        b = W.reshape(rows, cols // 32, 18)
        d = _f16(b[:, :, 0:2].copy()).reshape(rows, -1, 1)
        qs = b[:, :, 2:].astype(np.int64)
        vals = np.concatenate([(qs & 15) - 8, (qs >> 4) - 8], axis=2)
        return (vals * d).reshape(rows, cols)
    if wtype == Q8_0:
        b = W.reshape(rows, cols // 32, 34)
        d = _f16(b[:, :, 0:2].copy()).reshape(rows, -1, 1)
        qs = b[:, :, 2:].copy().view(np.int8).astype(np.float64)
        return (qs * d).reshape(rows, cols)
    if wtype == Q6_K:
        b = W.reshape(rows, cols // 256, 210)
        out = np.zeros((rows, cols // 256, 256))
        d = _f16(b[:, :, 208:210].copy())[:, :, 0]
        sc = b[:, :, 192:208].copy().view(np.int8).astype(np.float64)
        for h in range(2):
            ql = b[:, :, 64 * h:64 * h + 64].astype(np.int64)
            qh = b[:, :, 128 + 32 * h:128 + 32 * h + 32].astype(np.int64)
            for l in range(32):
                is_ = l // 16
                q = [(ql[:, :, l] & 15) | (((qh[:, :, l] >> 0) & 3) << 4),
                     (ql[:, :, l + 32] & 15) | (((qh[:, :, l] >> 2) & 3) << 4),
                     (ql[:, :, l] >> 4) | (((qh[:, :, l] >> 4) & 3) << 4),
                     (ql[:, :, l + 32] >> 4) | (((qh[:, :, l] >> 6) & 3) << 4)]
                for k in range(4):
                    out[:, :, 128 * h + l + 32 * k] = (d * sc[:, :, 8 * h + is_ + 2 * k]
                                                       * (q[k] - 32))
        return out.reshape(rows, cols)
    raise ValueError(wtype)


def matmul_truth(W, x, rows, cols, wtype):
    """float64 products and the per-row sum of |w x| (the error scale of an
    fp32 dot product in any summation order)."""
    A = dequant(W, wtype, rows, cols)
    xd = x.astype(np.float64)
    return A @ xd, np.abs(A) @ np.abs(xd)
