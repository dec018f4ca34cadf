"""Load-time preparation on the GPU (csrc/moek_prep.cu) against the torch restatement (prep.py, bit-exact against the
reference's own codec output in tests/golden): every output byte equal on the golden matrices (exception-rich, tiny
scales with scale factor 64, zeroed scales) and on seeded layers; the conversion time of a 512-expert layer."""
import numpy as np
import pytest
import torch

from qwen38_flash_coder_b200 import prep, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"
SETS = [("mw13", True), ("mw2", False), ("rw13", True), ("rw2", False), ("tw2", False)]


def _same(a: prep.PreparedMatrix, b: prep.PreparedMatrix):
    assert a.sf == b.sf
    for name in ("w", "sp", "g", "exc_off", "exc_ent"):
        x, y = getattr(a, name).cpu(), getattr(b, name).cpu()
        assert x.shape == y.shape and torch.equal(x, y), name


@pytest.mark.parametrize("name,gu", SETS)
def test_native_prep_matches_golden_matrices(golden, name, gu):
    if f"{name}_codes" not in golden:
        pytest.skip(f"{name}: no codes in the fixture")
    codes = torch.from_numpy(golden[f"{name}_codes"])
    scales = torch.from_numpy(golden[f"{name}_scales"]).view(torch.float8_e4m3fn)
    gs = torch.from_numpy(golden[f"{name}_gs"])
    nat = prep.PreparedMatrix(codes.to(DEV), scales.to(DEV), gs.to(DEV), gu)
    ref = prep.PreparedMatrix(codes, scales, gs, gu, native=False)
    _same(nat, ref)
    assert np.array_equal(nat.sp.cpu().numpy(), golden[f"{name}_tiled"])
    assert np.array_equal(nat.exc_ent.cpu().numpy(), golden[f"{name}_exc_ent"])


@pytest.mark.parametrize("e,h,i", [(64, 2048, 512), (16, 1024, 256)])
def test_native_prep_matches_torch_on_seeded_layers(e, h, i):
    w13, w2 = synth.make_layer(e, h, i, 3, device=DEV)
    for mat, gu in ((w13, True), (w2, False)):
        _same(prep.PreparedMatrix(*mat, gate_up=gu), prep.PreparedMatrix(*mat, gate_up=gu, native=False))


def test_native_prep_time_of_a_layer(capsys):
    """One 512-expert layer (hidden 2048, intermediate 512) converted by the kernels, timed with CUDA events."""
    w13, w2 = synth.make_layer(512, 2048, 512, 7, device=DEV)
    prep.PreparedLayer(w13, w2)  # warm-up (module load, allocations)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(3):
        prep.PreparedLayer(w13, w2)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / 3
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    prep.PreparedLayer(w13, w2, native=False)
    t1.record()
    torch.cuda.synchronize()
    with capsys.disabled():
        print(f"\nprep of one 512-expert layer: native {ms:.2f} ms, torch ops {t0.elapsed_time(t1):.2f} ms; "
              f"48 layers: {48 * ms / 1e3:.2f} s native")
    assert ms < 1000
