"""The kernels restate a few steps of the reference's arithmetic in cheaper but exactly equivalent
forms. These tests check each equivalence in IEEE float32 arithmetic (numpy rounds every float32
operation to nearest even, as the GPU's FP32 pipe does) on seeded and edge-case inputs."""
import numpy as np

f32 = np.float32
MAGIC = f32(12582912.0)  # 1.5 * 2^23


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def test_gelu_tail_saturate_form():
    """(x * 0.5) * (1 + clamp(t, -1, 1)) == x * sat(0.5 t + 0.5) (rowmath.cuh gelu_ref2)."""
    r = rng(0)
    t = np.concatenate([r.uniform(-1.5, 1.5, 400000), r.normal(0, 1, 100000), [-1, 1, -1.0000001, 1.0000001, 0]])
    t = np.concatenate([t, np.nextafter(f32(-1), f32(0)) + np.zeros(1), np.nextafter(f32(1), f32(2)) + np.zeros(1)]).astype(f32)
    x = (r.normal(0, 3, t.size) * np.exp(r.uniform(-20, 5, t.size))).astype(f32)
    ref = (x * f32(0.5)) * (f32(1) + np.clip(t, f32(-1), f32(1)))
    # fmaf(t, 0.5, 0.5): 0.5 t is exact, so one rounding of the sum
    v = np.clip(t * f32(0.5) + f32(0.5), f32(0), f32(1))
    got = x * v
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_quant_low_byte_and_range():
    """For |v| < 127.5, the low byte of bits(v + 1.5 * 2^23) is the half-even rounded int8, equal
    to the clamped form; and a row scaled by 127 / max|x| stays inside that range."""
    r = rng(1)
    v = np.concatenate([r.uniform(-127.49, 127.49, 500000), np.arange(-127, 128) + f32(0.5) * np.sign(np.arange(-127, 128))]).astype(f32)
    v = v[np.abs(v) < 127.5]
    bits = (v + MAGIC).view(np.uint32)
    low = (bits & 0xFF).astype(np.uint8).view(np.int8)
    ref = np.rint(np.clip(v, f32(-127), f32(127))).astype(np.int8)  # rint: half to even
    np.testing.assert_array_equal(low, ref)
    for seed in range(20):
        x = rng(100 + seed).normal(0, 10 ** rng(200 + seed).uniform(-6, 3), 1536).astype(f32)
        s = rng(300 + seed).uniform(0.5, 2, 1536).astype(f32)
        xs = x * s
        max_abs = np.maximum(np.abs(xs).max(), f32(1e-8))
        inv = f32(127) / max_abs
        assert np.abs(x * (s * inv)).max() < 127.5
        assert np.abs(xs * inv).max() < 127.5


def test_byte_perm_pack():
    """pack_i8x4: __byte_perm(__byte_perm(b0, b1, 0x40), __byte_perm(b2, b3, 0x40), 0x5410) puts
    the low bytes of b0..b3 in bytes 0..3 (selector nibbles index the 8 bytes of {b, a})."""
    def byte_perm(a, b, s):
        src = list(int(a).to_bytes(4, "little")) + list(int(b).to_bytes(4, "little"))
        return int.from_bytes(bytes(src[(s >> (4 * i)) & 7] for i in range(4)), "little")
    r = rng(2)
    for _ in range(2000):
        b = [int(x) for x in r.integers(0, 2**32, 4, dtype=np.uint64)]
        got = byte_perm(byte_perm(b[0], b[1], 0x0040), byte_perm(b[2], b[3], 0x0040), 0x5410)
        assert got == sum((b[i] & 0xFF) << (8 * i) for i in range(4))
