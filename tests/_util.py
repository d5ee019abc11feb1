"""Helpers shared by the tests: layout conversions between the oracle's NCHW
arrays and the device layouts of the C ABI (slab16 int8, slab8 fp16, NHWC fp16)."""
import numpy as np


def unsplit_columns(q: np.ndarray) -> np.ndarray:
    """Undo the stride-2 consumer layout: each row [even columns][odd columns] -> natural order."""
    wp = q.shape[3]
    out = np.empty_like(q)
    out[:, :, :, 0::2] = q[:, :, :, : wp // 2]
    out[:, :, :, 1::2] = q[:, :, :, wp // 2:]
    return out


def slab16_to_nchw(q: np.ndarray, c: int, h: int, w: int, stride: int = 1) -> np.ndarray:
    """[N][S][Hp][Wp][16] int8 -> [N][C][H][W] int8 (drops padding)."""
    if stride == 2:
        q = unsplit_columns(q)
    n, s, hp, wp, e = q.shape
    x = q.transpose(0, 1, 4, 2, 3).reshape(n, s * e, hp, wp)
    return np.ascontiguousarray(x[:, :c, :h, :w])


def nchw_to_nhwc(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x.transpose(0, 2, 3, 1))


def nhwc_to_nchw(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x.transpose(0, 3, 1, 2))


def silu_np(z):
    return z / (1.0 + np.exp(-z))


def seeded_act(rng, shape):
    """SiLU(N(0,1)) activations in fp16, the BASELINE input distribution."""
    return silu_np(rng.standard_normal(shape).astype(np.float32)).astype(np.float16)


def bits_to_f32(a) -> np.ndarray:
    return np.asarray(a).astype(np.int32).view(np.float32)
