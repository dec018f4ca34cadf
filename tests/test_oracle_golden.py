"""The CPU oracle against the golden fixtures made by running the reference's own Python (tests/golden/make_golden.py).

Mirrors the reference's CPU check (bench/moek/cpu_check.py: lossless scale round trip) and pins every oracle module
before any GPU result is compared with it.
"""
import numpy as np
import pytest
import torch

from oracle import align, marlin_scales, moe_ref, nvfp4, scale_codec

SETS = [("mw13", True), ("mw2", False), ("rw13", True), ("rw2", False), ("tw2", False)]


def test_e4m3_table_matches_torch():
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    ok = np.isnan(t) == np.isnan(nvfp4.E4M3)
    assert ok.all() and np.array_equal(t[~np.isnan(t)], nvfp4.E4M3[~np.isnan(t)])


def test_bf16_round_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 1e3
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(nvfp4.bf16_round(x), ref)


@pytest.mark.parametrize("name,gu", SETS)
def test_marlin_scale_bytes(golden, name, gu):
    sb, sf = marlin_scales.process_scales(golden[f"{name}_scales"])
    assert sf == golden[f"{name}_sf"][0]
    assert np.array_equal(sb, golden[f"{name}_sbytes"])
    g = marlin_scales.process_global(golden[f"{name}_gs"], sf)
    assert np.array_equal(g, golden[f"{name}_g"])


def test_logical_column_is_the_scale_permutation(golden):
    sb = golden["rw2_sbytes"][0]  # [K/16, N] processed
    ckpt = golden["rw2_scales"][0]  # [N, K/16] checkpoint bits
    n = sb.shape[1]
    cols = marlin_scales.logical_column(np.arange(n))
    # every processed byte is the S0E5M3 form of the checkpoint scale of its logical column
    vals = nvfp4.E4M3[ckpt[cols, :]].T  # [K/16, N]
    s0e5m3 = ((vals.astype(np.float16) * np.float16(128)).view(np.uint16).astype(np.uint32) >> 7) & 0xFF
    assert np.array_equal(sb, s0e5m3.astype(np.uint8))


@pytest.mark.parametrize("name,gu", SETS)
def test_pack_scales(golden, name, gu):
    packed, off, ent = scale_codec.pack_scales(golden[f"{name}_sbytes"], gu)
    assert np.array_equal(packed, golden[f"{name}_packed"])
    assert np.array_equal(off, golden[f"{name}_exc_off"])
    assert np.array_equal(ent, golden[f"{name}_exc_ent"])
    n = golden[f"{name}_sbytes"].shape[2]
    assert np.array_equal(scale_codec.tile_scales(packed, n, gu), golden[f"{name}_tiled"])


@pytest.mark.parametrize("name,gu", SETS)
def test_unpack_scales_round_trip(golden, name, gu):
    sb = golden[f"{name}_sbytes"]
    back = scale_codec.unpack_scales(golden[f"{name}_packed"], golden[f"{name}_exc_off"],
                                     golden[f"{name}_exc_ent"], sb.shape[1], sb.shape[2], gu)
    assert np.array_equal(back, sb)


def test_moe_reference_matches_problem_reference(golden):
    x = torch.from_numpy(golden["moe_x"]).view(torch.bfloat16)
    w13 = (golden["mw13_codes"], golden["mw13_scales"], golden["mw13_gs"])
    w2 = (golden["mw2_codes"], golden["mw2_scales"], golden["mw2_gs"])
    out = moe_ref.reference(x, golden["moe_ids"], golden["moe_wts"], w13, w2)
    ref = torch.from_numpy(golden["moe_out"])
    rel, _, _ = moe_ref.check(out, ref)
    assert rel < 1e-5, rel


def test_rounding_points(golden):
    """The kit kernel's rounding points stay within the reference's own 1e-2 bound (bench/moek/test_cuda.py:39) but
    not always within the 5e-3 gate; the oracle's points rounded once to bf16 (this build's kernels) do."""
    x = torch.from_numpy(golden["moe_x"]).view(torch.bfloat16)
    w13 = (golden["mw13_codes"], golden["mw13_scales"], golden["mw13_gs"])
    w2 = (golden["mw2_codes"], golden["mw2_scales"], golden["mw2_gs"])
    ref = torch.from_numpy(golden["moe_out"])
    kit = moe_ref.kit_semantics(x, golden["moe_ids"], golden["moe_wts"], w13, w2)
    rel, _, _ = moe_ref.check(kit, ref)
    assert rel <= 1e-2, rel
    mine = moe_ref.reference(x, golden["moe_ids"], golden["moe_wts"], w13, w2).to(torch.bfloat16)
    ok, stats = moe_ref.within_gate(mine, ref)
    assert ok and stats[2] == 0.0, stats  # a correctly rounded oracle has no error beyond half an ulp


def test_gate_net_of_output_rounding():
    r = torch.tensor([1.0, 3.0, 7.9, -6.0, 0.01])
    assert moe_ref.check(r.to(torch.bfloat16), r)[2] == 0.0
    bad = r.clone()
    bad[2] += 1.0
    assert moe_ref.check(bad, r)[2] > 0.2


def test_align_docstring_example(golden):
    sid, eid, npad = align.moe_align(golden["align_ids"], 4, 4)
    assert sid.size == 24 and int(npad[0]) == 16  # numel + E * (block - 1) entries; the docstring shows the prefix
    assert np.array_equal(sid[:16], golden["align_sorted"]) and (sid[16:] == 12).all()
    assert np.array_equal(eid, [0, 1, 2, 3, -1, -1])


def test_align_sizes_and_padding():
    rng = np.random.default_rng(1)
    for m, e, bs in ((1, 512, 96), (8, 512, 96), (3, 4, 16), (100, 64, 96), (7, 8, 8)):
        ids = np.stack([rng.choice(e, 5 if e >= 5 else e, replace=False) for _ in range(m)]).astype(np.int32)
        sid, eid, npad = align.moe_align(ids, e, bs)
        ls, lb = align.sizes(ids.size, e, bs)
        assert sid.size == ls and eid.size == lb
        n = int(npad[0])
        assert n % bs == 0 and (sid[n:] == ids.size).all()
        blocks = sid[:n].reshape(-1, bs)
        for b, row in enumerate(blocks):
            valid = row < ids.size
            assert valid[0] and (not valid.any() or valid[:valid.sum()].all())  # prefix, never empty
            assert (ids.reshape(-1)[row[valid]] == eid[b]).all()
        assert (eid[n // bs:] == -1).all()
        got = np.sort(sid[:n][sid[:n] < ids.size])
        assert np.array_equal(got, np.arange(ids.size))
