"""CPU oracle for the paged-KV write.  TEST INFRASTRUCTURE, NOT PRODUCT.

Only ``tests/`` may import this module, as the checker.  The product path
(``decodekernels_b200``) never imports it.

DecodeKernels has no cache-write kernel (its decode reads caches that vLLM's
``reshape_and_cache_flash`` wrote), so this restates that operation from its
definition:

* ``reshape_and_cache``: for every token ``t`` with
  ``slot = slot_mapping[t]`` in ``[0, num_blocks * block_size)``,
  ``cache[slot // bs, slot % bs, h, :] = x[t, h, :]`` for keys and values;
  negative slots (padding) and slots past the cache are skipped.
* ``e4m3_encode`` / ``e4m3_decode``: the OCP FP8 E4M3 ("fn": no infinities)
  format -- 1 sign bit, 4 exponent bits with bias 7, 3 mantissa bits;
  exponent field 0 holds subnormals ``m / 8 * 2**-6``; ``S.1111.111`` is NaN;
  the largest finite value is ``1.75 * 2**8 = 448``.  Encoding is
  round-to-nearest, ties to the even code, saturating finite values to
  +-448 (NaN stays NaN), applied to ``x / scale`` computed in float32 -- the
  convention of vLLM's per-tensor-scaled fp8 KV cache.

Parity pins: ``tests/test_cache_write_cpu.py`` checks the encoder against
torch's independent ``float8_e4m3fn`` conversion (with clamping) on random
values and every tie, subnormal and boundary case; on the GPU box
``tests/test_gpu_cache_write.py`` also compares the CUDA kernel with vLLM's
own ``reshape_and_cache_flash`` when vLLM's kernels load.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def _e4m3_table() -> np.ndarray:
    """float values of codes 0..127 (non-negative half; code 127 is NaN)."""
    vals = np.zeros(128, dtype=np.float64)
    for code in range(128):
        e, m = code >> 3, code & 7
        vals[code] = (m / 8.0) * 2.0**-6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
    vals[127] = np.nan
    return vals


_TABLE = _e4m3_table()
_FINITE = _TABLE[:127]  # codes 0..126, increasing


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """uint8 e4m3 codes -> float32."""
    c = np.asarray(codes, dtype=np.uint8)
    mag = _TABLE[c & 0x7F]
    return np.where(c & 0x80, -mag, mag).astype(np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> uint8 e4m3 codes: nearest, ties to even code, saturating."""
    x = np.asarray(x, dtype=np.float32)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.abs(x.astype(np.float64))
    nan = np.isnan(a)
    a = np.where(nan, 0.0, np.minimum(a, E4M3_MAX))
    hi = np.clip(np.searchsorted(_FINITE, a, side="left"), 0, 126)  # first code with value >= a
    lo = np.clip(hi - 1, 0, 126)
    d_hi = _FINITE[hi] - a
    d_lo = a - _FINITE[lo]
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & (lo % 2 == 0))
    code = np.where(pick_lo & (hi > 0), lo, hi).astype(np.uint8)
    code = np.where(nan, np.uint8(0x7F), code)
    return (code | sign).astype(np.uint8)


def quantize(x: np.ndarray, scale: float) -> np.ndarray:
    """Stored e4m3 codes of x with a per-tensor scale: e4m3(x / scale) in float32."""
    q = np.asarray(x, dtype=np.float32) / np.float32(scale)
    return e4m3_encode(q.astype(np.float32))


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, k_scale: float = 1.0,
                      v_scale: float = 1.0, fp8: bool = False) -> None:
    """Write key/value [T, Hkv, D] into the caches [blocks, bs, Hkv, D] (numpy
    arrays, modified in place; uint8 codes when ``fp8``)."""
    num_blocks, bs = key_cache.shape[0], key_cache.shape[1]
    slots = np.asarray(slot_mapping, dtype=np.int64)
    for t, slot in enumerate(slots):
        if slot < 0 or slot >= num_blocks * bs:
            continue
        b, o = divmod(int(slot), bs)
        if fp8:
            key_cache[b, o] = quantize(key[t], k_scale)
            value_cache[b, o] = quantize(value[t], v_scale)
        else:
            key_cache[b, o] = key[t]
            value_cache[b, o] = value[t]
