"""GGUF k-quant weight blocks as the attention projections use them.

kore stores every projection matrix in one of two GGUF block formats
(kore.cpp:322-381), 256 values per block along a row:

* Q4_K (type 12), 144 bytes: f16 d, f16 dmin, 12 bytes of packed 6-bit
  scales and mins for 8 sub-blocks of 32, 128 bytes of 4-bit values;
  value = d*scale*q - dmin*min.
* Q6_K (type 14), 210 bytes: 128 bytes of low 4 bits, 64 bytes of high 2
  bits, 16 int8 scales (one per 16 values), f16 d; value = d*scale*(q - 32).

``random_qmat`` builds seeded synthetic matrices in these layouts (every byte
pattern of the packed fields decodes, so random bytes with finite, scaled
f16 factors are valid weights), for tests and benchmarks: no checkpoint is
available offline.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

Q4_K = 12
Q6_K = 14
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}


@dataclass
class QMat:
    """A rows x cols matrix in GGUF blocks (row-major, cols a multiple of 256)."""
    type: int
    rows: int
    cols: int
    data: np.ndarray   # uint8 [rows * cols/256 * block bytes]

    def __post_init__(self):
        if self.type not in BLOCK_BYTES:
            raise ValueError(f"type {self.type} is neither Q4_K (12) nor Q6_K (14)")
        if self.cols % 256:
            raise ValueError(f"cols = {self.cols} is not a multiple of 256")
        self.data = np.ascontiguousarray(self.data, dtype=np.uint8).reshape(-1)
        if self.data.size != self.nbytes:
            raise ValueError(f"expected {self.nbytes} bytes, got {self.data.size}")

    @property
    def nbytes(self) -> int:
        return self.rows * (self.cols // 256) * BLOCK_BYTES[self.type]

    def row(self, r: int) -> np.ndarray:
        rb = (self.cols // 256) * BLOCK_BYTES[self.type]
        return self.data[r * rb:(r + 1) * rb]


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return np.asarray(v, np.float16).view(np.uint8).reshape(-1, 2)


def random_qmat(qtype: int, rows: int, cols: int, rng: np.random.Generator, sigma: float = 0.02) -> QMat:
    """Seeded synthetic weights with a standard deviation of roughly sigma."""
    nb = rows * (cols // 256)
    if qtype == Q4_K:
        b = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
        # E[sc*q] ~ 31.5*7.5, E[mn] ~ 31.5: d*270 ~ sigma, dmin ~ 7.5 d centres the values
        d = rng.uniform(0.75, 1.25, nb) * sigma / 270.0
        b[:, 0:2] = _f16_bytes(d)
        b[:, 2:4] = _f16_bytes(7.5 * d)
    elif qtype == Q6_K:
        b = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
        b[:, 192:208] = rng.integers(-127, 128, (nb, 16)).astype(np.int8).view(np.uint8)
        # E|sc*(q-32)| ~ 64*18: d ~ sigma / 1200
        d = rng.uniform(0.75, 1.25, nb) * sigma / 1200.0
        b[:, 208:210] = _f16_bytes(d)
    else:
        raise ValueError(f"type {qtype} is neither Q4_K (12) nor Q6_K (14)")
    return QMat(qtype, rows, cols, b.reshape(-1))
