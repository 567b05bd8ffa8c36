"""Bit-exact parity of the sm_100a kernels (through the libabx C ABI) with the oracle.

Models: the reference's SIMD-vs-scalar, chunk and thread-invariance checks
(tests/native/selftest.c:67-97, 240-336, 574-682) and tests/test_kernels.py:48-154, here
comparing the GPU against the CPU restatement of the reference at each SIMD rounding
pattern.  Every buffer -- master (fp32 or both fp24 planes), moments or FP8 codes and
scales, and the out copy -- must match bit for bit (NaN payloads excepted).
"""

from __future__ import annotations

import ctypes
import itertools

import numpy as np
import pytest
import torch

from conftest import device_segment, from_device, product_group, to_device
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ALGOS = (O.ADAMW, O.LION)
MOMENTS = (O.DT_F32, O.DT_BF16, O.DT_FP8)
MASTERS = (O.DT_F32, O.DT_F24)
GRADS = (O.DT_F32, O.DT_BF16)
OUTS = (O.DT_NONE, O.DT_F32, O.DT_BF16)
SIZES = (1, 37, 128, 129, 1000, 2049, 100003)

GROUP = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, seed=5)


def _run_steps(cases, kernels, oracle, level, steps=3, sr=1, g_scale=None, max_ctas=0):
    """Run ``steps`` updates of every case on the GPU (one multi_step call per step, all cases together) and
    in the oracle; return the list of (case description, mismatches)."""
    kernels.set_simd_level(O.SIMD_NAMES[level])
    gpu = [to_device(hs) for hs, _ in cases]
    ref = [hs.clone() for hs, _ in cases]
    pg = product_group(**GROUP, stochastic=sr)
    og = O.Group(**GROUP, stochastic=sr)
    scale_t = None if g_scale is None else torch.tensor([g_scale], dtype=torch.float32, device="cuda")
    for step in range(1, steps + 1):
        segs = []
        for (hs, _), dev, r in zip(cases, gpu, ref):
            hs.step = r.step = step
            r.new_grad(1000 * step + hs.n)
            dev["g"].copy_(torch.from_numpy(r.buffers["g"].view(np.int16) if r.buffers["g"].dtype == np.uint16
                                            else r.buffers["g"]).cuda())
            segs.append(device_segment(hs, dev, pg))
        arr = kernels.segment_array([ctypes.pointer(s) for s in segs])
        kernels.multi_step(None, arr, max_ctas, scale_t)
        osegs = [r.ctype(og) for r in ref]
        assert oracle.multi_step(osegs, level, g_scale) == 0
    torch.cuda.synchronize()
    results = []
    for (hs, desc), dev, r in zip(cases, gpu, ref):
        got = from_device(hs, dev)
        results.append((desc, got.mismatches(r)))
    return results


def _cases(seed0=0, sizes=SIZES, randomize=True):
    cases = []
    k = 0
    for algo, mv, pt, gt, ot in itertools.product(ALGOS, MOMENTS, MASTERS, GRADS, OUTS):
        for n in sizes:
            hs = O.HostSegment.random(n, gt, mv, ot, pt, algo, seed=seed0 + k, offset=128 * (k % 5), index=k)
            if randomize:
                hs.randomize_moments(seed0 + 7 * k)
            cases.append((hs, f"algo={algo} mv={mv} p={pt} g={gt} out={ot} n={n}"))
            k += 1
    return cases


@pytest.mark.parametrize("level", [O.SIMD_AVX512, O.SIMD_AVX2, O.SIMD_NEON, O.SIMD_SCALAR])
@pytest.mark.parametrize("sr", [1, 0])
def test_every_combination_bit_exact(kernels, oracle, level, sr):
    """All 72 dtype combinations x 7 sizes in one multi-segment call per step (several launches of up to 64
    segments each), 3 steps, nonzero starting moments."""
    bad = [(d, m) for d, m in _run_steps(_cases(), kernels, oracle, level, sr=sr) if m]
    assert not bad, f"{len(bad)} cases differ, e.g. {bad[:5]}"


def test_grad_scale_bit_exact(kernels, oracle):
    """The fused clip / unscale factor: g * s in fp32, rounded back to bf16 for bf16 gradients."""
    cases = _cases(seed0=11, sizes=(37, 2049))
    bad = [(d, m) for d, m in _run_steps(cases, kernels, oracle, O.SIMD_AVX512, g_scale=0.37) if m]
    assert not bad, bad[:5]


@pytest.mark.parametrize("sr", [1, 0])
def test_offsets_past_32_bits_bit_exact(kernels, oracle, sr):
    """Element offsets at and beyond 2^32 (a piece deep inside a huge tensor): the rounding streams index
    elements by the offset plus position modulo 2^32, as the reference does (csrc:100-106, 1577), so a piece
    whose indices wrap around 2^32 during the segment, and odd offsets (no 4-aligned hash groups) where the
    moments are not FP8, all match the oracle -- in partial tiles and in staged whole tiles."""
    cases = []
    k = 0
    for algo, mv, pt in itertools.product(ALGOS, MOMENTS, MASTERS):
        offsets = [(1 << 32) - 1024, (1 << 40) + (1 << 31) - 896, (1 << 33) + 384]
        if mv != O.DT_FP8:
            offsets += [(1 << 32) - 3, (1 << 35) + 1]
        for off in offsets:
            for n in (3000, 70001):
                hs = O.HostSegment.random(n, O.DT_BF16, mv, O.DT_BF16, pt, algo, seed=500 + k, offset=off, index=k)
                hs.randomize_moments(900 + k)
                cases.append((hs, f"algo={algo} mv={mv} p={pt} offset={off} n={n}"))
                k += 1
    bad = [(d, m) for d, m in _run_steps(cases, kernels, oracle, O.SIMD_AVX512, sr=sr) if m]
    assert not bad, f"{len(bad)} cases differ, e.g. {bad[:5]}"


def test_capped_grid_bit_exact(kernels, oracle):
    """max_ctas only changes which CTA takes which tile, never a result."""
    cases = _cases(seed0=3, sizes=(100003,))
    bad = [(d, m) for d, m in _run_steps(cases, kernels, oracle, O.SIMD_AVX512, max_ctas=3) if m]
    assert not bad, bad[:5]


@pytest.mark.parametrize("mv", MOMENTS)
@pytest.mark.parametrize("pt", MASTERS)
@pytest.mark.parametrize("algo", ALGOS)
def test_chunked_equals_whole(kernels, algo, mv, pt):
    """A tensor updated as 128-aligned chunks (segments with offsets) == updated whole, bit for bit
    (selftest.c:304-336): the property ZeRO-1 sharding relies on."""
    n = 300001
    cuts = [0, 65536, 131072 + 4096, n]
    hs = O.HostSegment.random(n, O.DT_BF16, mv, O.DT_BF16, pt, algo, seed=9).randomize_moments(4)
    whole, chunked = to_device(hs), to_device(hs)
    pg = product_group(**GROUP, stochastic=1)
    for step in (1, 2, 3):
        hs.step = step
        seg = device_segment(hs, whole, pg)
        kernels.multi_step(None, kernels.segment_array([ctypes.pointer(seg)]))
        parts = []
        for lo, hi in zip(cuts, cuts[1:]):
            # element views advanced to lo (FP8 codes are one byte per element; scales one per 128)
            sub = {k: (t[lo // 128:] if k in ("m_scale", "v_scale") else t[lo:]) for k, t in chunked.items()}
            part = O.HostSegment(hi - lo, hs.g_dtype, mv, hs.out_dtype, pt, algo, offset=lo, index=hs.index, step=step)
            parts.append(device_segment(part, sub, pg))
        kernels.multi_step(None, kernels.segment_array([ctypes.pointer(s) for s in parts]))
    torch.cuda.synchronize()
    for k in whole:
        assert torch.equal(whole[k], chunked[k]), k


def test_unaligned_buffers_take_the_scalar_path(kernels, oracle):
    """Buffers aligned to their element size but not to 16 bytes: the kernels fall back to element accesses
    and give the same bits."""
    n = 5000
    hs = O.HostSegment.random(n, O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.ADAMW, seed=2).randomize_moments(3)
    ref = hs.clone()
    big = {k: torch.zeros(t.numel() + 8, dtype=t.dtype, device="cuda") for k, t in to_device(hs).items()}
    dev = {k: big[k][1:1 + t.numel()] for k, t in to_device(hs).items()}
    for k, t in to_device(hs).items():
        dev[k].copy_(t)
    pg = product_group(**GROUP, stochastic=1)
    seg = device_segment(hs, dev, pg)
    kernels.set_simd_level("avx512")
    kernels.multi_step(None, kernels.segment_array([ctypes.pointer(seg)]))
    assert oracle.multi_step([ref.ctype(O.Group(**GROUP, stochastic=1))], O.SIMD_AVX512) == 0
    torch.cuda.synchronize()
    assert from_device(hs, dev).mismatches(ref) == {}


def test_misaligned_element_rejected(kernels):
    """A pointer not aligned to its element size is refused before launch (ABX_E_ALIGN)."""
    hs = O.HostSegment.random(64, O.DT_F32, O.DT_F32, O.DT_NONE, O.DT_F32, O.ADAMW, seed=1)
    dev = to_device(hs)
    seg = device_segment(hs, dev, product_group(**GROUP, stochastic=1))
    seg.m = dev["m"].data_ptr() + 2
    with pytest.raises(RuntimeError, match="code -21"):
        kernels.multi_step(None, kernels.segment_array([ctypes.pointer(seg)]))


def test_validation_codes_match_reference(kernels, oracle):
    """Every rejection code of check_segment (csrc:1537-1553) is returned before anything runs."""
    hs = O.HostSegment.random(256, O.DT_F32, O.DT_FP8, O.DT_BF16, O.DT_F32, O.ADAMW, seed=1)
    dev = to_device(hs)
    pg = product_group(**GROUP, stochastic=1)
    mutations = {
        "n": -1, "algorithm": 7, "p_dtype": 9, "g": None, "g_dtype": 3, "mv_dtype": 4, "out_dtype": 3,
        "out": None, "m_scale": None, "offset": 100, "group": None,
    }
    for field, value in mutations.items():
        seg = device_segment(hs, dev, pg)
        setattr(seg, field, value)
        oseg = hs.ctype(O.Group(**GROUP, stochastic=1))
        setattr(oseg, field, value)
        want = oracle.check_segment(oseg, True)
        rc = kernels._lib.abx_multi_step(None, kernels.segment_array([ctypes.pointer(seg)]), 1, 0)
        assert rc == want != 0, (field, rc, want)
    before = {k: t.clone() for k, t in dev.items()}
    good = device_segment(hs, dev, pg)
    bad = device_segment(hs, dev, pg)
    bad.g = None
    rc = kernels._lib.abx_multi_step(None, kernels.segment_array([ctypes.pointer(good), ctypes.pointer(bad)]), 2, 0)
    torch.cuda.synchronize()
    assert rc == -2
    assert all(torch.equal(before[k], dev[k]) for k in dev), "a rejected call must update nothing"


def test_fused_adamw_entry_point(kernels, oracle):
    """abx_fused_adamw (the single-tensor entry, csrc:1518) == multi_apply with the same coefficients."""
    from adambridge_b200 import native
    n = 4099
    rng = np.random.default_rng(0)
    p = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    g = torch.from_numpy((rng.standard_normal(n) * 1e-3).astype(np.float32)).cuda().bfloat16()
    m = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    c = native.StepCoefficients.for_step(1e-3, 0.9, 0.999, 1e-8, 0.01, 1)
    hp = kernels.make_hparams(c, 1234, True)
    hs = O.HostSegment(n, O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.ADAMW)
    hs.buffers = {"p": p.cpu().numpy().copy(), "g": g.view(torch.int16).cpu().numpy().view(np.uint16).copy(),
                  "m": np.zeros(n, np.uint16), "v": np.zeros(n, np.uint16), "out": np.zeros(n, np.uint16)}
    kernels.set_simd_level("avx512")
    kernels.fused_adamw(p, g, m, v, out, hp, 0, n)
    ohp = O.HParams(*[getattr(hp, f) for f, _ in O.HParams._fields_])
    assert oracle.multi_apply([hs.ctype()], [ohp], O.SIMD_AVX512) == 0
    torch.cuda.synchronize()
    assert np.array_equal(p.cpu().numpy().view(np.uint32), hs.buffers["p"].view(np.uint32))
    assert np.array_equal(m.view(torch.int16).cpu().numpy().view(np.uint16), hs.buffers["m"])
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), hs.buffers["out"])


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("n,at", [(1024, 0), (8192, 0), (8192, 4096)])
def test_fp8_specials(kernels, oracle, algo, n, at):
    """Saturating values, zero blocks, subnormal-range moments and infinite block maxima through the FP8
    codec (the encode / decode pair of csrc:826-876), against the oracle -- in a partial tile (read from
    HBM directly) and in whole staged tiles (the fast path)."""
    hs = O.HostSegment.random(n, O.DT_F32, O.DT_FP8, O.DT_F32, O.DT_F32, algo, seed=5)
    g = hs.buffers["g"]
    g[at:at + 128] = 0.0                                    # a block whose m stays 0: scale 1
    g[at + 128:at + 256] = np.float32(1e-30) * np.arange(128)   # tiny: subnormal codes after scaling
    g[at + 256:at + 384] = np.float32(3e38)                 # huge: maxima overflow to inf in v
    g[at + 384] = np.float32(np.inf)                        # infinite m: block scale inf / 448 = inf
    g[at + 385] = -np.float32(np.inf)
    dev = to_device(hs)
    ref = hs.clone()
    pg = product_group(**GROUP, stochastic=1)
    kernels.set_simd_level("avx512")
    kernels.multi_step(None, kernels.segment_array([ctypes.pointer(device_segment(hs, dev, pg))]))
    assert oracle.multi_step([ref.ctype(O.Group(**GROUP, stochastic=1))], O.SIMD_AVX512) == 0
    torch.cuda.synchronize()
    got = from_device(hs, dev)
    # NaN codes may differ in sign (the sign of a NaN is not specified); compare everything else exactly
    for k in ("m", "v") if algo == O.ADAMW else ("m",):
        a, b = got.buffers[k], ref.buffers[k]
        nan_a = (a & 0x7F) >= (0x7F if k == "m" else 0x7D)
        nan_b = (b & 0x7F) >= (0x7F if k == "m" else 0x7D)
        assert np.array_equal(nan_a, nan_b), k
        assert np.array_equal(a[~nan_a], b[~nan_b]), k
    for k in ("p", "out", "m_scale", "v_scale") if algo == O.ADAMW else ("p", "out", "m_scale"):
        a, b = got.buffers[k], ref.buffers[k]
        same = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
        assert same.all(), (k, np.flatnonzero(~same)[:10])


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("sr", [1, 0])
def test_fp8_codec_wide_dynamic_range(kernels, oracle, algo, sr):
    """FP8 moments whose block scales span 1e-30 .. 1e10 and gradients spanning 1e-30 .. 1e3: blocks on both
    sides of the reciprocal-division range, subnormal and saturated codes, every code value.  Bit-exact with the
    oracle (which divides and encodes exactly as the reference does)."""
    n = 1 << 20
    hs = O.HostSegment.random(n, O.DT_F32, O.DT_FP8, O.DT_BF16, O.DT_F32, algo, seed=77)
    rng = np.random.default_rng(78)
    nb = hs.nblocks
    hs.buffers["m"][:] = rng.integers(0, 256, hs.moment_len(), dtype=np.uint8)
    hs.buffers["m"][(hs.buffers["m"] & 0x7F) == 0x7F] = 0x11          # no NaN codes in the starting state
    hs.buffers["m_scale"][:] = np.exp(rng.uniform(np.log(1e-30), np.log(1e10), nb)).astype(np.float32)
    if algo == O.ADAMW:
        hs.buffers["v"][:] = rng.integers(0, 0x7C, hs.moment_len(), dtype=np.uint8)
        hs.buffers["v_scale"][:] = np.exp(rng.uniform(np.log(1e-30), np.log(1e10), nb)).astype(np.float32)
    kernels.set_simd_level("avx512")
    dev = to_device(hs)
    ref = hs.clone()
    pg = product_group(**GROUP, stochastic=sr)
    og = O.Group(**GROUP, stochastic=sr)
    for step in (1, 2, 3):
        g = (np.sign(rng.standard_normal(n)) * np.exp(rng.uniform(np.log(1e-30), np.log(1e3), n))).astype(np.float32)
        ref.buffers["g"][:] = g
        dev["g"].copy_(torch.from_numpy(g).cuda())
        hs.step = ref.step = step
        kernels.multi_step(None, kernels.segment_array([ctypes.pointer(device_segment(hs, dev, pg))]))
        assert oracle.multi_step([ref.ctype(og)], O.SIMD_AVX512) == 0
    torch.cuda.synchronize()
    assert from_device(hs, dev).mismatches(ref) == {}


def test_pipeline_status_clear_after_all_updates(kernels):
    """No bounded pipeline wait gave up in any update of this session (the status word is still zero)."""
    assert kernels.pipeline_status() == 0


@pytest.mark.parametrize("prec", [O.DT_BF16, O.DT_FP8])
def test_ema_stall_known_answer(kernels, oracle, prec):
    """The reference's EMA-stall known answer (tests/test_precision.py:99-123) through the GPU kernel: 500 steps of
    v <- 0.999 v + 0.001 g^2 (AdamW with b1 = 0, g^2 = 1.5 every step, v starting at 1).  Round-to-nearest
    moments freeze at 1 (bf16) or near it (FP8); stochastic rounding tracks the exact EMA (~1.197).  Every step
    runs on the GPU and in the oracle, and the final second moments agree bit for bit."""
    n = 4096
    target = np.full(n, 1.5, np.float32)
    target[::128] = 4.0          # one larger value per block, so FP8 block scales stay put
    tracked = np.ones(n, bool)
    tracked[::128] = False
    kernels.set_simd_level("scalar")
    try:
        results = _ema_runs(kernels, oracle, prec, n, target, tracked)
    finally:
        kernels.set_simd_level(None)
    exact = 1.5 + (1.0 - 1.5) * 0.999 ** 500
    assert results[0] == pytest.approx(1.0, abs=1e-6) if prec == O.DT_BF16 else results[0] < 1.1
    assert results[1] == pytest.approx(exact, rel=0.01 if prec == O.DT_BF16 else 0.03)


def _ema_runs(kernels, oracle, prec, n, target, tracked):
    from adambridge_b200 import native
    results = {}
    for sr in (0, 1):
        hs = O.HostSegment.random(n, O.DT_F32, prec, O.DT_NONE, O.DT_F32, O.ADAMW, seed=1)
        hs.buffers["g"][:] = np.sqrt(target)
        init = np.ones(n, np.float32)
        init[::128] = 4.0
        if prec == O.DT_BF16:
            hs.buffers["v"][:] = O.bf16_bits(init)
        else:
            scale = np.float32(2.0) / np.float32(57344.0)
            hs.buffers["v_scale"][:] = scale
            hs.buffers["v"][:] = [oracle.fp8_encode(float(np.float32(x / scale)), 0, 0, "v") for x in np.sqrt(init)]
        dev = to_device(hs)
        arr = kernels.segment_array([ctypes.pointer(device_segment(hs, dev))])
        for step in range(1, 501):
            seed = oracle.step_seed(0, 0, step)
            h = O.HParams(0.0, 0.999, 1.0, np.float32(1 - 0.999), 1.0, 0.0, 1.0, 1e-8, seed, sr)
            kernels.multi_apply(None, arr, [native._HParams(*[getattr(h, f) for f, _ in O.HParams._fields_])])
            assert oracle.multi_apply([hs.ctype()], [h], O.SIMD_SCALAR) == 0
        got = from_device(hs, dev)
        assert not got.mismatches(hs), got.mismatches(hs)
        if prec == O.DT_BF16:
            v = O.bf16_to_f32(got.buffers["v"])
        else:
            v = np.array([oracle.fp8_decode(int(c), "v") for c in got.buffers["v"][:n]], np.float32)
            v = (v * np.repeat(got.buffers["v_scale"], 128)[:n]) ** 2
        results[sr] = float(v[tracked].mean())
    return results
