"""Seeded synthetic inputs shared by the parity tests (numpy, CPU)."""
import numpy as np

BB = {12: 144, 13: 176, 14: 210}


def f16_bits(a):
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def random_blocks(rng, ggml_type, nblocks, scale=0.02):
    """Uniform random bytes with |N(0, scale)| fp16 d (and dmin) fields."""
    bb = BB[ggml_type]
    b = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    d = f16_bits(np.abs(rng.normal(0, scale, nblocks)))
    if ggml_type == 14:
        b[:, 208] = d & 0xFF
        b[:, 209] = d >> 8
    else:
        dm = f16_bits(np.abs(rng.normal(0, scale, nblocks)))
        b[:, 0] = d & 0xFF
        b[:, 1] = d >> 8
        b[:, 2] = dm & 0xFF
        b[:, 3] = dm >> 8
    return b.reshape(-1)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def d2h_f32(ptr, n):
    """n float32 values at a raw device address (a buffer the library allocated)."""
    from cuda.bindings import runtime as rt
    host = np.empty(n, np.float32)
    err, = rt.cudaMemcpy(host.ctypes.data, ptr, n * 4, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert int(err) == 0, err
    return host
