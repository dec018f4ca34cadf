"""Load-time weight preparation (qwen38_flash_coder_b200.prep) against the golden fixtures and the CPU oracle.

Mirrors the reference's CPU-side checks (bench/moek/cpu_check.py: the packed-scale round trip) and its tiled ==
plain check (bench/moek/test_tiled.py:12-15) for this build's own weight layout.
"""
import numpy as np
import pytest
import torch

from oracle import marlin_scales
from qwen38_flash_coder_b200 import prep, synth

SETS = [("mw13", True), ("mw2", False), ("rw13", True), ("rw2", False), ("tw2", False)]


def _scales(golden, name):
    return torch.from_numpy(golden[f"{name}_scales"]).view(torch.float8_e4m3fn)


@pytest.mark.parametrize("name,gu", SETS)
def test_marlin_bytes_and_global(golden, name, gu):
    s = _scales(golden, name)
    sf = prep.scale_factor(s)
    assert sf == golden[f"{name}_sf"][0]
    assert np.array_equal(prep.marlin_scale_bytes(s, sf).numpy(), golden[f"{name}_sbytes"])
    g = prep.global_scale(torch.from_numpy(golden[f"{name}_gs"]), sf)
    assert np.array_equal(g.numpy(), golden[f"{name}_g"])


@pytest.mark.parametrize("name,gu", SETS)
def test_pack_scales_bit_exact(golden, name, gu):
    sb = torch.from_numpy(golden[f"{name}_sbytes"])
    for chunk in (32, 3):  # expert chunking must not change the result
        packed, off, ent = prep.pack_scales(sb, gu, chunk=chunk)
        assert np.array_equal(packed.numpy(), golden[f"{name}_packed"])
        assert np.array_equal(off.numpy(), golden[f"{name}_exc_off"])
        assert np.array_equal(ent.numpy(), golden[f"{name}_exc_ent"])
    n = sb.shape[2]
    assert np.array_equal(prep.tile_scales(packed, n, gu).numpy(), golden[f"{name}_tiled"])


def test_pack_scales_no_exceptions():
    sb = torch.full((2, 16, 256), 0x90, dtype=torch.uint8)
    packed, off, ent = prep.pack_scales(sb, False)
    assert int(off[-1]) == 0 and ent.numel() == 1 and int(ent[0]) == 0
    assert (packed[..., :16] == 0x90).all() and (packed[..., 16:] == 0).all()


@pytest.mark.parametrize("gate_up,n,k", [(True, 512, 256), (False, 256, 512), (True, 1024, 128)])
def test_tile_weights_round_trip(gate_up, n, k):
    g = torch.Generator().manual_seed(n + k)
    codes = torch.randint(0, 256, (3, n, k // 2), dtype=torch.uint8, generator=g)
    w = prep.tile_weights(codes, gate_up)
    assert w.shape == (3, k // 16, 2 * n) and w.dtype == torch.int32
    assert torch.equal(prep.untile_weights(w, n, gate_up), codes)


def test_tile_weights_word_contents():
    """Spot-check the documented layout: word w of row r in the block of (item t, stage s), halves swizzled."""
    n, k = 512, 256
    codes = torch.randint(0, 256, (1, n, k // 2), dtype=torch.uint8, generator=torch.Generator().manual_seed(3))
    w = prep.tile_weights(codes, True).view(-1)
    cols = prep.item_columns(n, True)
    rng = np.random.default_rng(0)
    for _ in range(300):
        t, s, r, wd = (int(rng.integers(x)) for x in (n // 256, k // 64, 256, 8))
        pos = (((wd >> 2) ^ ((r >> 2) & 1)) << 2) | (wd & 3)
        word = int(w[((t * (k // 64) + s) * 256 + r) * 8 + pos]) & 0xFFFFFFFF
        col = int(cols[t, r])
        for i in range(8):
            kk = 64 * s + 8 * wd + i
            byte = int(codes[0, col, kk // 2])
            code = (byte >> 4) if kk & 1 else (byte & 15)
            assert sum(((word >> bp) & 1) << b for b, bp in enumerate(prep.CODE_BITS[i])) == code


def test_quantizer_matches_reference_e2m1(golden):
    x = torch.from_numpy(golden["e2m1_in"])
    mag = torch.bucketize(x.abs().clamp(max=6.0), synth._MIDS, right=False)
    codes = (mag | ((x < 0).to(mag.dtype) << 3)).to(torch.uint8)
    assert torch.equal(codes, torch.from_numpy(golden["e2m1_codes"]))


def test_quantizer_scales_and_dequant_error():
    w = (torch.randn((2, 64, 256), generator=torch.Generator().manual_seed(1)) * 0.02).to(torch.bfloat16)
    codes, scales, gs = synth.quantize_nvfp4(w)
    assert codes.shape == (2, 64, 128) and scales.shape == (2, 64, 16) and gs.shape == (2,)
    assert float(scales.float().max()) <= 448.0
    from oracle.nvfp4 import dequant_expert

    for e in range(2):
        deq = dequant_expert(codes[e].numpy(), scales[e].view(torch.uint8).numpy(), float(gs[e]))
        rel = np.linalg.norm(deq - w[e].float().numpy()) / np.linalg.norm(w[e].float().numpy())
        assert rel < 0.12, rel  # NVFP4 on Gaussian weights: ~9 % relative error


def test_oracle_logical_column_matches_device_permutation():
    """The device helper slot_position/position_slot pair is the inverse of oracle.marlin_scales.logical_column."""
    pos = np.arange(128)
    slot = marlin_scales.logical_column(pos)  # slot within the 128-run of each position
    inv = np.empty(128, dtype=np.int64)
    inv[slot] = pos
    # restate the device arithmetic of moek_common.cuh in Python
    def slot_position(s):
        c = s & 63
        m = 8 * (c & 7) + (c >> 3)
        r = m & 3
        return (s & 64) | (m & ~3) | (2 if r == 1 else 1 if r == 2 else r)

    assert all(slot_position(s) == inv[s] for s in range(128))


def test_prepared_layer_bytes():
    w13 = synth.make_experts(4, 512, 256, 1)
    w2 = synth.make_experts(4, 256, 256, 2)
    layer = prep.PreparedLayer(w13, w2)
    per = layer.expert_bytes()
    assert per.shape == (4,)
    total = layer.w13.nbytes() + layer.w2.nbytes()
    assert abs(int(per.sum()) - total) <= 8 * 4  # offsets: E*keys + 1 per matrix


def test_unsupported_shapes_raise():
    with pytest.raises(ValueError):
        prep.check_shapes(300, 256, False)
    with pytest.raises(ValueError):
        prep.check_shapes(512, 200, True)


def test_device_pair_decode_matches_code_bits():
    """The device's word decode (moek_common.cuh fp4_pairs: a mask, two rotate-and-masks, a two-part gather),
    restated here, yields for pair p the codes 2p and 2p + 1 of prep.CODE_BITS at the bf16 positions (sign 15, e1 e0 m
    at 8..6; the same 16 bits higher for the second code)."""
    rotr = lambda q, n: ((q >> n) | (q << (32 - n))) & 0xFFFFFFFF
    P = 0x81C081C0

    def pairs(q):
        return [q & P, rotr(q, 4) & P, rotr(q, 10) & P, (rotr(q, 14) & 0x00400040) | (rotr(q, 6) & 0x81808180)]

    def place(code):  # m, e0, e1 at 6, 7, 8 and the sign at 15
        return (code & 7) << 6 | ((code >> 3) & 1) << 15

    flat = [b for bits in prep.CODE_BITS for b in bits]
    assert sorted(flat) == list(range(32))
    rng = np.random.default_rng(7)
    for _ in range(2000):
        codes = [int(c) for c in rng.integers(0, 16, 8)]
        q = sum(((c >> b) & 1) << pos for c, bits in zip(codes, prep.CODE_BITS) for b, pos in enumerate(bits))
        for p, d in enumerate(pairs(q)):
            assert d == place(codes[2 * p]) | place(codes[2 * p + 1]) << 16


def test_device_small_division_restated():
    """The layer kernel's div_small (fp32 reciprocal estimate of v / d, one correction each way) restated with an
    fp32 reciprocal of the same accuracy as the hardware's approximate one (relative error 2^-23): exact for every
    v < 2^22 and d < 2^10 that the unit plan and unit decode use (sampled, plus the extremes)."""
    rng = np.random.default_rng(3)
    v = np.concatenate([rng.integers(0, 1 << 22, 200000), np.arange(0, 5000), [(1 << 22) - 1] * 10])
    d = np.concatenate([rng.integers(1, 1 << 10, 200000), rng.integers(1, 65, 5000), np.arange(1, 11)])
    for err in (-2.0 ** -23, 0.0, 2.0 ** -23):  # the reciprocal's worst relative errors either way
        r = (np.float32(1.0) / d.astype(np.float32)) * np.float32(1.0 + err)
        q = np.trunc(v.astype(np.float32) * r.astype(np.float32)).astype(np.int64)
        rem = v - q * d
        q += (rem >= d).astype(np.int64) - (rem < 0).astype(np.int64)
        assert np.array_equal(q, v // d)
