"""Parity of every CUDA kernel with the oracle, on a B200. Run with: pytest -m gpu.

Tolerance (written here, applied by oracle.check_close): |y - ref| <= min(1e-2 * rms(ref), 1e-2)
+ 1e-2 * |ref|, i.e. both the reference's rule (int4gemv/reference.py:13-22) and the tier's
rtol = atol = 1e-2. Unpack and dequantize are compared bit for bit.
"""

import numpy as np
import pytest
import torch

import oracle
from int4gemv import ops

pytestmark = pytest.mark.gpu
RTOL = 1e-2
ATOL = 1e-2

KERNELS = [
    ("naive", {}),
    ("coalesced", {}),
    ("vectorized", {}),
    ("vectorized", {"threads_per_block": 256, "rows_per_warp": 1}),
    ("vectorized", {"threads_per_block": 64, "rows_per_warp": 4}),
    ("w4a16", {}),
]
FAST = ["stripe_mma", "tc_dequant", "stream_mma", "tcgen05", "mma_pipeline"]


def stripe_fits(m, n, k):
    """stripe_plan's shared-memory rule: the fewest K-panels (1, 2, 4, ...; one for M <= 2) whose
    permuted x (17 bytes per 8 weights, per-item padded), tables and warp partials leave room for
    three 34 KB stripes in 227 KB."""
    if m > 8 or k % 2048:
        return False
    units = (n + 3) // 4
    rows_cap = 4 * (-(-units // min(torch.cuda.get_device_properties(0).multi_processor_count,
                                    units)))
    stripes = k // 2048
    mc = m if m <= 2 else 4 if m <= 4 else 8
    ts = 2 if m <= 2 else mc
    panels = 1
    while panels <= stripes and (m > 2 or panels == 1):
        items = -(-stripes // panels) * 16
        xs = items * 272
        if mc == 8:
            xs += (64 - xs % 128 + 128) % 128
        off = 1536 + m * xs + items * 4 * ts * 4 + items * ts * 4 + 16 * rows_cap * mc * 4
        off = -(-off // 1024) * 1024
        if off < 227 * 1024 and (227 * 1024 - off) // 34816 >= 3:
            return True
        panels *= 2
    return False


def expected_kernel(m, k, g=128, n=8192):
    """The kernel int4gemv_w4a16 picks on the fast path's shapes: stripe_mma for M <= 8 and K a
    multiple of 2048 when its x panels fit (stripe_fits); tc_dequant for 9 <= M <= 64; stream_mma
    for the rest (M <= 32, K a multiple of 1024)."""
    if g != 128:
        return "stream_mma"
    if 9 <= m <= 64 and k % 1024 == 0:
        return "tc_dequant"
    return "stripe_mma" if stripe_fits(m, n, k) else "stream_mma"


def cuda(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def run(name, cfg, args, g):
    y = getattr(ops, name)(*args, g, **cfg)
    torch.cuda.synchronize()
    return y


def assert_close(y, ref, what=""):
    ok, msg = oracle.check_close(y.float().cpu().numpy() if isinstance(y, torch.Tensor) else y,
                                 ref, RTOL, ATOL)
    assert ok, f"{what}: {msg}"


@pytest.mark.parametrize("name,cfg", KERNELS, ids=[f"{n}{c}" for n, c in KERNELS])
def test_golden(golden, name, cfg):
    g = int(golden["group_size"])
    args = cuda(golden["x"], golden["qweight"], golden["scales"], golden["zeros"])
    if name == "vectorized" and g % 32 != 0:
        with pytest.raises(RuntimeError, match="group_size must be a multiple of 32"):
            run(name, cfg, args, g)
        return
    y = run(name, cfg, args, g)
    assert y.dtype == torch.float16 and tuple(y.shape) == golden["y_ref"].shape
    assert_close(y, golden["y_ref"], f"{golden['name']} vs reference.py")
    ref64 = oracle.reference(golden["x"], golden["qweight"], golden["scales"], golden["zeros"], g)
    assert_close(y, ref64, f"{golden['name']} vs oracle")


def test_unpack_dequantize_bit_exact(golden):
    g = int(golden["group_size"])
    qw, s, z = cuda(golden["qweight"], golden["scales"], golden["zeros"])
    q = ops.unpack(qw).cpu().numpy()
    np.testing.assert_array_equal(q, oracle.unpack(golden["qweight"]))
    w = ops.dequantize(qw, s, z, g).cpu().numpy()
    want = golden["deq"] if "deq" in golden else oracle.dequantize(
        golden["qweight"], golden["scales"], golden["zeros"], g)
    np.testing.assert_array_equal(w.view(np.uint32), want.view(np.uint32))


# BASELINE.json configs at full size: M = 1 shapes, the M sweep, and the full sharded shapes.
FULL = [
    (1, 4096, 4096), (1, 8192, 8192), (1, 14336, 4096), (1, 4096, 14336),
    (2, 8192, 8192), (4, 8192, 8192), (8, 8192, 8192), (16, 8192, 8192), (32, 8192, 8192),
    (1, 28672, 8192), (1, 8192, 28672), (8, 28672, 8192), (8, 8192, 28672),
]


@pytest.mark.parametrize("m,n,k", FULL, ids=[f"m{m}_n{n}_k{k}" for m, n, k in FULL])
def test_full_size_w4a16(m, n, k):
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=m + n + k)
    args = cuda(x, q, s, z)
    y = ops.w4a16(*args, 128)
    ref = oracle.reference(x, q, s, z, 128)
    kernel = ops.w4a16_kernel(*args, 128)
    assert_close(y, ref, f"w4a16 {m}x{n}x{k} ({kernel})")
    assert kernel == expected_kernel(m, k, n=n)
    # The margin: the largest error as a fraction of the allowed bound. Measured on B200 at these
    # shapes: at most 0.05 for the warp-MMA kernels (the fp16 rounding of y) up to K = 28672, and
    # 0.35 for tc_dequant (weights rounded to fp16); half the budget is the alarm.
    yf = y.float().cpu().numpy().astype(np.float64)
    bound = min(ATOL * float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))), ATOL) + RTOL * np.abs(ref)
    ratio = float((np.abs(yf - ref) / bound).max())
    assert ratio < 0.5, f"w4a16 {m}x{n}x{k} ({kernel}): error uses {ratio:.2f} of the tolerance"


@pytest.mark.parametrize("name,cfg", KERNELS[:3] + [("w4a16", {})])
def test_config0_all_kernels(name, cfg):
    x, q, s, z = oracle.synthetic(1, 4096, 4096, 128, seed=0)
    y = run(name, cfg, cuda(x, q, s, z), 128)
    assert_close(y, oracle.reference(x, q, s, z), name)
    # and against the reference's own CPU path, bit-exact oracle of csrc/sequential.cpp
    assert_close(y, oracle.sequential(x, q, s, z).astype(np.float32), name + " vs sequential")


ODD = [
    (1, 1, 256, 128), (1, 7, 384, 128), (3, 17, 640, 128), (5, 149, 1024, 64), (9, 150, 512, 32),
    (16, 300, 2048, 128), (13, 37, 768, 256), (2, 148 * 130 + 5, 1024, 128), (1, 64, 8192, 128),
    (7, 5000, 1152, 128), (12, 256, 4096, 128), (1, 19000, 256, 32), (2, 333, 896, 64),
]


@pytest.mark.parametrize("m,n,k,g", ODD, ids=[f"m{m}_n{n}_k{k}_g{g}" for m, n, k, g in ODD])
def test_ragged_shapes(m, n, k, g):
    x, q, s, z = oracle.synthetic(m, n, k, g, seed=n * 7 + k)
    args = cuda(x, q, s, z)
    ref = oracle.reference(x, q, s, z, g)
    for name, cfg in KERNELS:
        assert_close(run(name, cfg, args, g), ref, f"{name}{cfg}")


def fast_kernels_for(args, g):
    """The fast kernels that accept this shape (the others raise a clear error)."""
    out = []
    for kern in FAST:
        try:
            y = ops.w4a16_with(*args, g, kern)
            torch.cuda.synchronize()
            out.append((kern, y))
        except RuntimeError as e:
            assert kern in str(e)
    return out


@pytest.mark.parametrize("m,n,k,g", ODD + [(m, n, k, 128) for m, n, k in FULL],
                         ids=[f"m{m}_n{n}_k{k}_g{g}" for m, n, k, g in ODD] +
                             [f"m{m}_n{n}_k{k}_g128" for m, n, k in FULL])
def test_each_fast_kernel(m, n, k, g):
    x, q, s, z = oracle.synthetic(m, n, k, g, seed=n + 3 * k + m)
    args = cuda(x, q, s, z)
    ref = oracle.reference(x, q, s, z, g)
    for kern, y in fast_kernels_for(args, g):
        assert_close(y, ref, f"{kern} {m}x{n}x{k} g{g}")


def test_fast_kernel_coverage():
    """stream_mma and tc_dequant take every BASELINE shape (stripe_mma those with M <= 2);
    mma_pipeline takes group 32 / 64."""
    x, q, s, z = cuda(*oracle.synthetic(1, 256, 8192, 128))
    assert [k for k, _ in fast_kernels_for([x, q, s, z], 128)] == FAST
    x, q, s, z = cuda(*oracle.synthetic(2, 256, 1024, 32))
    assert [k for k, _ in fast_kernels_for([x, q, s, z], 32)] == ["mma_pipeline"]


# stream_mma edge cases: rows per CTA that leave a 16-row tile empty or partly filled, N not a
# multiple of 4, every M tile count (1..4 tiles of 8 rows of x, partly filled), and K large
# enough (for the M) that x is taken in several k-panels, including a shorter last panel.
STREAM = [
    (1, 1, 1024), (1, 5, 1024), (3, 33, 2048), (8, 17, 3072), (9, 100, 1024), (17, 301, 2048),
    (24, 64, 1024), (31, 148 * 4 + 3, 1024), (32, 4099, 8192), (16, 8192, 14336),
    (8, 1000, 28672), (1, 14336, 16384), (2, 4096, 32768), (5, 148 * 36 + 2, 5120),
    (12, 777, 7168), (1, 148 * 28, 1024),
]


@pytest.mark.parametrize("m,n,k", STREAM, ids=[f"m{m}_n{n}_k{k}" for m, n, k in STREAM])
def test_stream_mma_shapes(m, n, k):
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=11 * m + n + k)
    args = cuda(x, q, s, z)
    assert ops.w4a16_kernel(*args, 128) == expected_kernel(m, k, n=n)
    y = ops.w4a16_with(*args, 128, "stream_mma")
    torch.cuda.synchronize()
    assert_close(y, oracle.reference(x, q, s, z, 128), f"stream_mma {m}x{n}x{k}")


# stripe_mma edge cases: rows per CTA below one 16-row tile, between one and two tiles, several
# 32-row blocks, N not a multiple of 4, M = 1 to 8 (M = 3 and 4: two groups x four rows of x per
# MMA, M = 3 with an empty column; M = 5..8: one group x eight rows), K from one stripe (2048) to
# 28672, one or several K-panels of x.
STRIPE = [
    (1, 1, 2048), (2, 5, 2048), (1, 37, 8192), (2, 148 * 4 + 3, 4096), (1, 148 * 20 + 1, 6144),
    (2, 148 * 24, 2048), (1, 148 * 36 + 2, 10240), (2, 4099, 8192), (1, 1000, 28672),
    (2, 300, 14336), (1, 28672, 2048), (3, 1, 2048), (4, 37, 8192), (3, 148 * 4 + 3, 4096),
    (4, 4099, 8192), (3, 8192, 8192), (4, 14336, 4096), (4, 148 * 36 + 2, 6144),
    # K-panels (x prepared one panel at a time) and the MC = 8 layout (M = 5..8)
    (4, 4096, 14336), (3, 1000, 28672), (5, 37, 2048), (6, 4099, 4096), (7, 148 * 4 + 3, 8192),
    (8, 8192, 8192), (8, 4096, 14336), (5, 14336, 4096), (8, 1000, 28672), (8, 148 * 36 + 2, 6144),
]


@pytest.mark.parametrize("m,n,k", STRIPE, ids=[f"m{m}_n{n}_k{k}" for m, n, k in STRIPE])
def test_stripe_mma_shapes(m, n, k):
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=13 * m + n + k)
    args = cuda(x, q, s, z)
    assert ops.w4a16_kernel(*args, 128) == expected_kernel(m, k, n=n)
    y = ops.w4a16_with(*args, 128, "stripe_mma")
    torch.cuda.synchronize()
    assert_close(y, oracle.reference(x, q, s, z, 128), f"stripe_mma {m}x{n}x{k}")


def test_stripe_mma_rejects():
    """Shapes stripe_mma does not take raise a clear error when it is asked for by name."""
    for m, k, why in ((9, 2048, r"M must be in \[1, 8\]"), (1, 3072, "K must be a multiple of 2048")):
        args = cuda(*oracle.synthetic(m, 64, k, 128))
        with pytest.raises(RuntimeError, match=why):
            ops.w4a16_with(*args, 128, "stripe_mma")


# tc_dequant edge cases: N not a multiple of the 128-row tile (rows past N read as zeros), a single
# tile shared by many CTAs (K large, N small: up to 112 contributors per tile), ranges that cover
# whole tiles, every accumulator width (M rounded up to 16, 32, 48, 64) with partly filled rows of
# x, K from one 1024-weight block to 28672, and N beyond 148 tiles.
TD = [
    (1, 1, 1024), (9, 37, 1024), (16, 100, 28672), (17, 128, 1024), (24, 129, 2048),
    (32, 148 * 128 + 3, 1024), (33, 1000, 4096), (48, 300, 3072), (64, 4096, 2048),
    (64, 129, 8192), (40, 8192, 8192), (12, 28672, 8192), (20, 4096, 14336), (10, 14336, 4096),
    (2, 148 * 128 * 2 + 77, 2048), (63, 3000, 5120),
]


@pytest.mark.parametrize("m,n,k", TD, ids=[f"m{m}_n{n}_k{k}" for m, n, k in TD])
def test_tc_dequant_shapes(m, n, k):
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=17 * m + n + k)
    args = cuda(x, q, s, z)
    assert ops.w4a16_kernel(*args, 128) == expected_kernel(m, k, n=n)
    y = ops.w4a16_with(*args, 128, "tc_dequant")
    torch.cuda.synchronize()
    assert_close(y, oracle.reference(x, q, s, z, 128), f"tc_dequant {m}x{n}x{k}")
    y2 = ops.w4a16_with(*args, 128, "tc_dequant")
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "tc_dequant must be deterministic (fixed-order split-K sums)"


def test_tc_dequant_rejects():
    """Shapes tc_dequant does not take raise a clear error when it is asked for by name."""
    for m, k, g, why in ((65, 1024, 128, r"M must be in \[1, 64\]"),
                         (4, 1536, 128, "K must be a positive multiple of 1024"),
                         (4, 1024, 64, "group_size must be 128")):
        args = cuda(*oracle.synthetic(m, 64, k, g))
        with pytest.raises(RuntimeError, match=why):
            ops.w4a16_with(*args, g, "tc_dequant")


def test_tc_dequant_two_streams():
    """tc_dequant's split-K partial sums and tile counters live in static device memory; calls
    issued on two streams without any synchronisation between them are ordered by the library
    (an event between the streams), so every result stays correct."""
    m, n, k = 16, 4096, 4096
    sets = [oracle.synthetic(m, n, k, 128, seed=300 + i) for i in range(6)]
    dev = [cuda(*st) for st in sets]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    outs = []
    for i, args in enumerate(dev):
        with torch.cuda.stream(streams[i % 2]):
            outs.append(ops.w4a16_with(*args, 128, "tc_dequant"))
    torch.cuda.synchronize()
    for i, (x, q, s, z) in enumerate(sets):
        assert_close(outs[i], oracle.reference(x, q, s, z, 128), f"call {i}")


# tc_wide: 256-row tiles and 64-weight stages, so other tile / range boundaries than
# tc_dequant's: N one row past a tile, N below one tile, K long enough for several s/z windows per
# CTA (16 stages each), contributors per tile from one to hundreds, every M up to 64 (rows of x
# past M in the last 8-row group).
TW = [(1, 1, 1024), (9, 37, 1024), (16, 100, 28672), (33, 1000, 4096), (48, 300, 3072),
      (63, 3000, 5120), (16, 8192, 8192), (64, 8192, 8192), (16, 257, 1024),
      (9, 148 * 256 + 1, 1024), (5, 512, 28672), (64, 255, 4096), (1, 256, 1024)]


@pytest.mark.parametrize("m,n,k", TW, ids=[f"m{m}_n{n}_k{k}" for m, n, k in TW])
def test_tc_wide_shapes(m, n, k):
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=29 * m + n + k)
    args = cuda(x, q, s, z)
    y = ops.w4a16_with(*args, 128, "tc_wide")
    torch.cuda.synchronize()
    assert_close(y, oracle.reference(x, q, s, z, 128), f"tc_wide {m}x{n}x{k}")
    y2 = ops.w4a16_with(*args, 128, "tc_wide")
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "tc_wide must be deterministic (fixed-order split-K sums)"
    from int4gemv import capi

    assert capi.device_status() == 0


def test_tc_wide_two_streams():
    """Like tc_dequant, tc_wide's partial sums and tile counters are static; calls on two streams
    with no synchronisation between them are ordered by the library."""
    m, n, k = 16, 4096, 4096
    sets = [oracle.synthetic(m, n, k, 128, seed=400 + i) for i in range(6)]
    dev = [cuda(*st) for st in sets]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    outs = []
    for i, args in enumerate(dev):
        with torch.cuda.stream(streams[i % 2]):
            outs.append(ops.w4a16_with(*args, 128, "tc_wide"))
    torch.cuda.synchronize()
    for i, (x, q, s, z) in enumerate(sets):
        assert_close(outs[i], oracle.reference(x, q, s, z, 128), f"call {i}")


@pytest.mark.parametrize("m,n,k,g", [(1, 2048, 3584, 128), (3, 300, 768, 64), (2, 100, 96, 16),
                                     (12, 257, 1536, 128)])
def test_w4a16_f32_any_shape(m, n, k, g):
    """The fp32 row sums off the fast path's shapes (a K shard of a split layer need not be a
    multiple of 1024): the SIMT kernels store fp32."""
    x, q, s, z = oracle.synthetic(m, n, k, g, seed=7 + m + k)
    y = ops.w4a16_f32(*cuda(x, q, s, z), g)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    assert_close(y.cpu().numpy(), oracle.reference(x, q, s, z, g), f"w4a16_f32 {m}x{n}x{k} g{g}")


@pytest.mark.parametrize("m,n,k", [(9, 1000, 2048), (16, 4096, 8192), (64, 300, 1024)])
def test_w4a16_f32_tc_dequant(m, n, k):
    """The fp32 row sums (the K-split partials of a sharded layer) through tc_dequant."""
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=5 + m)
    y = ops.w4a16_f32(*cuda(x, q, s, z), 128)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    assert_close(y.cpu().numpy(), oracle.reference(x, q, s, z, 128), f"w4a16_f32 M={m}")


@pytest.mark.parametrize("kern,m", [("stripe_mma", 1), ("stripe_mma", 2), ("stripe_mma", 3),
                                    ("stripe_mma", 4), ("stripe_mma", 8), ("stream_mma", 1),
                                    ("stream_mma", 2), ("stream_mma", 8), ("stream_mma", 16),
                                    ("tcgen05", 1), ("tc_dequant", 1), ("tc_dequant", 16),
                                    ("tc_dequant", 40)])
def test_repeated_calls_weights_in_l2(kern, m):
    """The same weights (34 MB, resident in the 126 MB L2 after the first call) in eight calls in a
    row: every ring refill then lands within a few hundred nanoseconds, so a stage released before
    its shared-memory loads have returned would be overwritten under them. Each call is checked."""
    x, q, s, z = oracle.synthetic(m, 8192, 8192, 128, seed=41 + m)
    args = cuda(x, q, s, z)
    ref = oracle.reference(x, q, s, z, 128)
    for rep in range(8):
        y = ops.w4a16_with(*args, 128, kern)
        torch.cuda.synchronize()
        assert_close(y, ref, f"{kern} M={m} call {rep}")


def test_strict_weights_after_in_place_requantise():
    """Weights written by the kernel right before the GEMV in the same stream (device quantize in
    place) with int4gemv_set_strict_weights(1): the GEMV waits for them, on every fast kernel; the
    strict and default orderings give bit-identical results when nothing writes the weights."""
    from int4gemv import capi

    lib = capi.lib()
    for m, k, kern in ((1, 4096, "stripe_mma"), (2, 4096, "stripe_mma"), (4, 4096, "stripe_mma"),
                       (3, 4096, "stream_mma"),
                       (12, 2048, "stream_mma"), (1, 1024, "tcgen05"), (16, 2048, "tc_dequant"),
                       (33, 1024, "tc_dequant")):
        n = 2048
        gen = torch.Generator(device="cuda").manual_seed(m * k)
        w0 = torch.randn(n, k, generator=gen, device="cuda") * 0.02
        w1 = torch.randn(n, k, generator=gen, device="cuda") * 0.02
        x = torch.randn(m, k, generator=gen, device="cuda").half()
        q, s, z = ops.quantize(w0, 128)
        y_default = ops.w4a16_with(x, q, s, z, 128, kern)
        capi.check(lib.int4gemv_set_strict_weights(1))
        try:
            y_strict = ops.w4a16_with(x, q, s, z, 128, kern)
            assert torch.equal(y_default.view(torch.int16), y_strict.view(torch.int16)), kern
            for _ in range(3):  # re-quantise in place, then multiply right after it
                q1, s1, z1 = ops.quantize(w1, 128)
                q.copy_(q1)
                s.copy_(s1)
                z.copy_(z1)
                y = ops.w4a16_with(x, q, s, z, 128, kern)
                torch.cuda.synchronize()
                want = oracle.reference(x.cpu().numpy(), q1.cpu().numpy(), s1.cpu().numpy(),
                                        z1.cpu().numpy(), 128)
                assert_close(y, want, f"strict {kern} M={m}")
                w0, w1 = w1, w0
        finally:
            capi.check(lib.int4gemv_set_strict_weights(0))


def test_stream_mma_chained_calls():
    """Back-to-back launches overlap (programmatic stream serialization): each GEMV reads the
    previous one's output as x, so an early read of x or a late write of y shows up here. Every
    layer is checked against the oracle run on that layer's actual input."""
    n = 4096
    rng = np.random.default_rng(3)
    layers = [oracle.synthetic(1, n, n, 128, seed=100 + i)[1:] for i in range(6)]
    dev_layers = [cuda(q, s, z) for q, s, z in layers]
    for rep in range(3):
        x0 = (rng.standard_normal((2, n)) * 0.5).astype(np.float16)
        hs = [cuda(x0)[0]]
        for q, s, z in dev_layers:
            hs.append(ops.w4a16(hs[-1], q, s, z, 128))
        torch.cuda.synchronize()
        for i, (q, s, z) in enumerate(layers):
            h_in = hs[i].cpu().numpy()
            assert_close(hs[i + 1], oracle.reference(h_in, q, s, z, 128), f"rep {rep} layer {i}")
    assert capi_status() == 0


def capi_status():
    from int4gemv import capi
    return capi.device_status()


def test_group_sizes_without_fast_path():
    # group 8 and 16: only naive / coalesced / w4a16 (which falls back) apply
    for g in (8, 16, 24):
        x, q, s, z = oracle.synthetic(3, 40, 96 * (g // 8), g, seed=g)
        args = cuda(x, q, s, z)
        ref = oracle.reference(x, q, s, z, g)
        for name in ("naive", "coalesced", "w4a16"):
            assert_close(run(name, {}, args, g), ref, f"{name} g={g}")
        assert ops.w4a16_kernel(*args, g) == "coalesced"


def test_empty_and_zero_k():
    for name, cfg in KERNELS:
        x = torch.zeros(0, 256, dtype=torch.float16, device="cuda")
        q = torch.zeros(8, 32, dtype=torch.int32, device="cuda")
        s = torch.ones(8, 2, dtype=torch.float16, device="cuda")
        assert run(name, cfg, (x, q, s, s), 128).shape == (0, 8)
        x = torch.zeros(3, 256, dtype=torch.float16, device="cuda")
        assert run(name, cfg, (x, q[:0], s[:0], s[:0]), 128).shape == (3, 0)
        x = torch.zeros(3, 0, dtype=torch.float16, device="cuda")
        q0 = torch.zeros(8, 0, dtype=torch.int32, device="cuda")
        s0 = torch.zeros(8, 0, dtype=torch.float16, device="cuda")
        y = run(name, cfg, (x, q0, s0, s0), 128)
        assert y.shape == (3, 8) and bool((y == 0).all())


def test_misaligned_inputs():
    x, q, s, z = oracle.synthetic(2, 64, 512, 128, seed=5)
    xs = torch.empty(x.size + 8, dtype=torch.float16, device="cuda")
    xs = xs[1:1 + x.size].view(2, 512)  # 2-byte aligned only
    xs.copy_(torch.from_numpy(x))
    args = [xs] + cuda(q, s, z)
    ref = oracle.reference(x, q, s, z)
    assert ops.w4a16_kernel(*args, 128) == "coalesced"
    assert_close(run("w4a16", {}, args, 128), ref, "w4a16 misaligned x")
    assert_close(run("naive", {}, args, 128), ref, "naive misaligned x")
    with pytest.raises(RuntimeError, match="x and qweight must be 16-byte aligned"):
        run("vectorized", {}, args, 128)


@pytest.mark.parametrize("m", [1, 3, 4, 16, 40])
def test_deterministic(m):
    x, q, s, z = oracle.synthetic(m, 8192, 8192, 128, seed=11)
    args = cuda(x, q, s, z)
    a = ops.w4a16(*args, 128)
    b = ops.w4a16(*args, 128)
    assert torch.equal(a, b)


def test_noncontiguous_and_device_checks():
    x, q, s, z = cuda(*oracle.synthetic(2, 64, 256, 128))
    with pytest.raises(RuntimeError, match="w4a16: inputs must be contiguous"):
        ops.w4a16(x, q.T.contiguous().T, s, z, 128)
    with pytest.raises(RuntimeError, match="expected all inputs on one cuda device"):
        ops.w4a16(x, q, s.cpu(), z, 128)


def test_register_limit_message():
    with pytest.raises(RuntimeError, match=r"vectorized: this configuration uses \d+ registers per "
                                           r"thread, so blocks of at most \d+ threads fit, not 1024"):
        x, q, s, z = cuda(*oracle.synthetic(8, 64, 256, 128))
        ops.vectorized(x, q, s, z, 128, threads_per_block=1024, rows_per_warp=4)


def load_only_oracle(x, q, s, z, g):
    """out[r] = XOR of row r's words, of its scale / zero bit patterns (once per group), and of
    the x words read with every 32-weight chunk."""
    n, words = q.shape
    k = words * 8
    xw = np.ascontiguousarray(x[0]).view(np.uint32).reshape(k // 32, 16)
    x_per_chunk = np.bitwise_xor.reduce(xw, axis=1)
    x_all = np.bitwise_xor.reduce(x_per_chunk)
    out = np.bitwise_xor.reduce(q.view(np.uint32), axis=1)
    out ^= x_all
    out ^= np.bitwise_xor.reduce(s.view(np.uint16).astype(np.uint32), axis=1)
    out ^= np.bitwise_xor.reduce(z.view(np.uint16).astype(np.uint32), axis=1)
    return out


@pytest.mark.parametrize("tpb,rpw", [(128, 2), (32, 1), (256, 4)])
def test_load_only(tpb, rpw):
    x, q, s, z = oracle.synthetic(1, 333, 1024, 128, seed=2)
    out = ops.load_only(*cuda(x, q, s, z), 128, threads_per_block=tpb, rows_per_warp=rpw)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), load_only_oracle(x, q, s, z, 128))


def test_kernel_info():
    for name, info in ops.KERNEL_INFO.items():
        d = info(1)
        assert set(d) == {"registers", "local_bytes", "threads_per_block", "max_threads_per_block",
                          "blocks_per_sm", "warps_per_sm"}
        assert d["registers"] > 0 and d["blocks_per_sm"] >= 1, (name, d)
    d = ops.KERNEL_INFO["vectorized"](8, threads_per_block=256, rows_per_warp=4)
    assert d["threads_per_block"] == 256


def test_matches_reference_gpu_kernels():
    """The reference's own CUDA kernels, built from its sources for sm_100a, agree with ours."""
    import importlib.util
    from pathlib import Path
    so = sorted((Path(__file__).resolve().parents[1] / "oracle" / "_ref").glob("int4gemv_ref*.so"))
    if not so:
        pytest.skip("reference not built (oracle/_ref)")
    spec = importlib.util.spec_from_file_location("int4gemv_ref", so[0])
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    for m in (1, 8):
        x, q, s, z = oracle.synthetic(m, 4096, 4096, 128, seed=m)
        args = cuda(x, q, s, z)
        theirs = ref.vectorized(*args, 128).float().cpu().numpy()
        assert_close(theirs, oracle.reference(x, q, s, z), "reference vectorized vs oracle")
        ours = ops.w4a16(*args, 128).float().cpu().numpy()
        assert_close(ours, oracle.reference(x, q, s, z), "w4a16 vs oracle")
        assert np.max(np.abs(ours - theirs)) <= 0.02 * (1 + np.max(np.abs(theirs)))


def test_device_status_clean():
    from int4gemv import capi
    assert capi.device_status() == 0


# Fused gate / up projection: silu(x @ gate^T) * (x @ up^T) from one interleaved weight stream.
SILU = [(1, 4096, 4096), (2, 512, 1024), (4, 1000, 2048), (8, 4102, 3072), (17, 300, 1024),
        (32, 1024, 8192), (1, 14336, 4096)]


@pytest.mark.parametrize("m,n,k", SILU, ids=[f"m{m}_n{n}_k{k}" for m, n, k in SILU])
def test_silu_mul(m, n, k):
    from int4gemv import quant

    x, qg, sg, zg = oracle.synthetic(m, n, k, 128, seed=5 * n + k)
    _, qu, su, zu = oracle.synthetic(m, n, k, 128, seed=5 * n + k + 1)
    gate = oracle.reference(x, qg, sg, zg, 128).astype(np.float64)
    up = oracle.reference(x, qu, su, zu, 128).astype(np.float64)
    want = gate / (1.0 + np.exp(-gate)) * up
    q, s, z = (quant.interleave_rows(*cuda(a, b)) for a, b in ((qg, qu), (sg, su), (zg, zu)))
    y = ops.w4a16_silu_mul(cuda(x)[0], q, s, z, 128)
    torch.cuda.synchronize()
    assert tuple(y.shape) == (m, n)
    assert_close(y, want.astype(np.float32), f"silu_mul {m}x{n}x{k}")


def test_silu_mul_rejects():
    x, q, s, z = cuda(*oracle.synthetic(1, 6, 1024, 128))
    with pytest.raises(RuntimeError, match="pairs"):
        ops.w4a16_silu_mul(x, q[:5], s[:5], z[:5], 128)
    x, q, s, z = cuda(*oracle.synthetic(1, 8, 512, 128))
    with pytest.raises(RuntimeError, match="K must be a multiple of 1024"):
        ops.w4a16_silu_mul(x, q, s, z, 128)


# Fused bias / residual epilogue: y = x @ W^T + bias + residual, rounded to fp16 once, on every
# kernel the dispatcher can pick (the shapes below reach stripe_mma, tc_dequant, stream_mma,
# mma_pipeline, vectorized and coalesced).
BIAS = [(1, 8192, 8192, 128, "stripe_mma"), (2, 1000, 4096, 128, "stripe_mma"),
        (4, 1000, 2048, 128, "stripe_mma"),
        (5, 300, 1024, 128, "stream_mma"), (16, 1000, 2048, 128, "tc_dequant"),
        (40, 300, 1024, 128, "tc_dequant"),
        (3, 257, 768, 64, "mma_pipeline"), (2, 100, 640, 128, "vectorized"),
        (4, 77, 96, 16, "coalesced")]


@pytest.mark.parametrize("m,n,k,g,kernel", BIAS, ids=[f"{b[4]}_m{b[0]}_n{b[1]}" for b in BIAS])
@pytest.mark.parametrize("with_bias,with_res", [(True, True), (True, False), (False, True)])
def test_bias_residual(m, n, k, g, kernel, with_bias, with_res):
    x, q, s, z = oracle.synthetic(m, n, k, g, seed=n + k + g)
    rng = np.random.default_rng(m * n)
    bias = rng.standard_normal(n).astype(np.float16)
    res = rng.standard_normal((m, n)).astype(np.float16)
    want = oracle.reference(x, q, s, z, g).astype(np.float64)
    if with_bias:
        want = want + bias.astype(np.float64)
    if with_res:
        want = want + res.astype(np.float64)
    args = cuda(x, q, s, z)
    assert ops.w4a16_kernel(*args, g) == kernel
    tb, tr = cuda(bias, res)
    y = ops.w4a16_bias_residual(*args, g, bias=tb if with_bias else None,
                                residual=tr if with_res else None)
    torch.cuda.synchronize()
    assert_close(y, want.astype(np.float32), f"{kernel} bias={with_bias} residual={with_res}")


def test_bias_residual_in_place_and_empty():
    """residual may be y itself (through the C ABI); K = 0 gives bias + residual; M = 0 is empty."""
    from int4gemv import capi

    m, n, k = 2, 4096, 4096
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=9)
    rng = np.random.default_rng(9)
    bias = rng.standard_normal(n).astype(np.float16)
    res = rng.standard_normal((m, n)).astype(np.float16)
    tx, tq, ts, tz, tb, ty = cuda(x, q, s, z, bias, res)
    stream = torch.cuda.current_stream().cuda_stream
    capi.call("int4gemv_w4a16_bias_residual", ty.data_ptr(), tx.data_ptr(), tq.data_ptr(),
              ts.data_ptr(), tz.data_ptr(), tb.data_ptr(), ty.data_ptr(), m, n, k, 128, stream)
    torch.cuda.synchronize()
    want = oracle.reference(x, q, s, z, 128).astype(np.float64) + bias + res.astype(np.float64)
    assert_close(ty, want.astype(np.float32), "in place")

    x0 = torch.empty(m, 0, dtype=torch.float16, device="cuda")
    q0 = torch.empty(n, 0, dtype=torch.int32, device="cuda")
    s0 = torch.empty(n, 0, dtype=torch.float16, device="cuda")
    tr = cuda(res)[0]
    y = ops.w4a16_bias_residual(x0, q0, s0, s0, 128, bias=tb, residual=tr)
    torch.cuda.synchronize()
    want0 = (bias.astype(np.float32) + res.astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint16), want0.view(np.uint16))
    assert ops.w4a16_bias_residual(tx[:0], tq, ts, tz, 128, bias=tb).shape == (0, n)
    with pytest.raises(RuntimeError, match="bias must be"):
        ops.w4a16_bias_residual(tx, tq, ts, tz, 128, bias=tb[:-1])
    with pytest.raises(RuntimeError, match="residual must be"):
        ops.w4a16_bias_residual(tx, tq, ts, tz, 128, residual=tr.t())


# Grouped launch: matrices sharing x, weights stacked by rows, one output per matrix.
GROUPED = [(1, [4096, 1024, 1024], 4096, 128), (4, [4096, 1024, 1024], 4096, 128),
           (17, [300, 5, 0, 77], 2048, 128), (2, [14336, 14336], 4096, 128),
           (3, [200, 96], 768, 64)]


@pytest.mark.parametrize("m,sizes,k,g", GROUPED,
                         ids=[f"m{m}_{'-'.join(map(str, s))}_k{k}_g{g}" for m, s, k, g in GROUPED])
def test_grouped(m, sizes, k, g):
    from int4gemv import quant

    x = oracle.synthetic(m, 8, k, g, seed=m)[0]
    mats = [oracle.synthetic(1, max(n, 1), k, g, seed=100 * i + n)[1:] for i, n in enumerate(sizes)]
    mats = [tuple(t[:n] for t in mat) for mat, n in zip(mats, sizes)]
    stacked = [quant.stack_rows(*cuda(*(mat[j] for mat in mats))) for j in range(3)]
    ys = ops.w4a16_grouped(cuda(x)[0], *stacked, g, sizes)
    torch.cuda.synchronize()
    assert len(ys) == len(sizes)
    for (q, s, z), n, y in zip(mats, sizes, ys):
        assert tuple(y.shape) == (m, n)
        if n:
            assert_close(y, oracle.reference(x, q, s, z, g), f"grouped matrix of {n} rows")


def test_grouped_rejects():
    x, q, s, z = cuda(*oracle.synthetic(1, 64, 1024, 128))
    with pytest.raises(RuntimeError, match="add up to"):
        ops.w4a16_grouped(x, q, s, z, 128, [32, 16])
    with pytest.raises(RuntimeError, match="between 1 and 8"):
        ops.w4a16_grouped(x, q, s, z, 128, [8] * 8 + [0])
