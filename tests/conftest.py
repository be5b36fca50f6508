"""Shared test setup: import paths, the `gpu` marker, seeded input generators."""
from __future__ import annotations

import os
import sys
import zlib

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "encoding-experiment_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def pytest_collection_modifyitems(config, items):
    """A bound on every test (pytest-timeout, thread method: it also ends a test stuck inside a C call), so a
    hung host call fails the run instead of holding the GPU until an outer limit."""
    try:
        import pytest_timeout  # noqa: F401
    except ImportError:
        return
    for item in items:
        if item.get_closest_marker("timeout") is None:
            item.add_marker(pytest.mark.timeout(600, method="thread"))


def seed_for(*parts) -> int:
    """Deterministic seed from a config / matrix / layer name."""
    return zlib.crc32("/".join(str(p) for p in parts).encode()) & 0x7FFFFFFF


def normal(seed: int, n: int, std: float = 1.0) -> np.ndarray:
    """f32 ~ N(0, std) from numpy PCG64 (np.random.default_rng)."""
    return np.random.default_rng(seed).standard_normal(n, dtype=np.float32) * np.float32(std)


def lcg_synth(n: int, seed: int, inc: int = 1442695040888963407) -> np.ndarray:
    """The reference tests' LCG in [-1, 1) (crates/larql-compute/tests/test_q4_x86_correctness.rs:73-79;
    inc=1 gives tests/test_metal_shaders.rs:18-24)."""
    out = np.empty(n, np.float32)
    s = seed
    m = (1 << 64) - 1
    for i in range(n):
        s = (s * 6364136223846793005 + inc) & m
        out[i] = np.float32((s >> 33)) / np.float32(4294967295.0) * np.float32(2.0) - np.float32(1.0)
    return out


def random_f16_bits(rng, n: int, lo_exp: int = -20, hi_exp: int = 2) -> np.ndarray:
    """Finite random f16 values with random sign and exponent in [lo_exp, hi_exp]."""
    mant = rng.uniform(1.0, 2.0, n)
    ex = rng.integers(lo_exp, hi_exp + 1, n)
    sign = rng.choice([-1.0, 1.0], n)
    return (sign * mant * np.exp2(ex)).astype(np.float16).view(np.uint16)


def random_q4k_blocks(seed: int, rows: int, hidden: int, signed_scales: bool = True) -> np.ndarray:
    """Random-byte LARQL Q4_K rows: every nibble value, every 6-bit scale, random finite f16 d/dmin."""
    rng = np.random.default_rng(seed)
    nsb = rows * hidden // 256
    b = rng.integers(0, 256, size=(nsb, 148), dtype=np.uint8)
    d = random_f16_bits(rng, nsb)
    dm = random_f16_bits(rng, nsb)
    if not signed_scales:
        d &= 0x7FFF
        dm &= 0x7FFF
    b[:, 0:2] = d.view(np.uint8).reshape(nsb, 2)
    b[:, 2:4] = dm.view(np.uint8).reshape(nsb, 2)
    return b.reshape(-1)


def max_err_ok(got: np.ndarray, ref: np.ndarray, rel: float = 1e-3):
    """max |err| <= rel * ||ref||_inf."""
    err = float(np.max(np.abs(got.astype(np.float64) - ref.astype(np.float64)))) if ref.size else 0.0
    bound = rel * float(np.max(np.abs(ref))) if ref.size else 0.0
    return err <= bound, err, bound


@pytest.fixture(scope="session")
def backend():
    import larql_cuda
    b = larql_cuda.CudaBackend(0)
    yield b
    b.close()
