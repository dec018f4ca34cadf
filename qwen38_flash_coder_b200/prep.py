"""Load-time conversion of checkpoint NVFP4 experts into the kernels' layouts: this build's prep kernels on a CUDA
device (csrc/moek_prep.cu, ``PreparedMatrix``), and the same conversion restated with torch ops below (the CPU path,
and the kernels' test reference).

Input: the checkpoint tensors vLLM hands to ``prepare_nvfp4_moe_layer_for_marlin`` (vllm/.../marlin_utils_fp4.py:
288-298): ``weight`` uint8 [E, N, K/2] (element 2i in the low nibble), ``weight_scale`` float8 E4M3 [E, N, K/16],
``weight_scale_2`` fp32 [E].

Output, per matrix:

- **scales**: vLLM's Marlin scale bytes (marlin_utils_fp4.py:30-146,355-386: shared power-of-two factor, the 64-value
  ``scale_perm`` and the [0, 2, 1, 3] pair swap, the S0E5M3 byte), then the kit's lossless packed format and item
  tiling (files/mbx_moek.py:61-172). The byte format is the reference's, bit for bit; the code is this module's own
  (window choice by pairwise counting instead of sort + searchsorted).
- **global scale**: ``weight_scale_2 * 2^119 / scale_factor`` (marlin_utils_fp4.py:134-146,385-386).
- **weights**: this build's tiled layout, an int32 tensor of the reference's shape [E, K/16, 2N] (same bytes as the
  checkpoint, reordered). Per (expert, 256-row item, 64-k stage) one contiguous 8 KB block of 256 rows x 32 bytes:
  row r holds the item's row r over the stage's 64 k as 8 words, word w = the 8 consecutive k ``64s + 8w + i``
  (i = 0..7), so words 2c and 2c + 1 are k-group c (one scale). Inside a word the 4 bits of code i (m, e0, e1, sign
  = bits 0..3 of the E2M1 code) sit at bit positions ``CODE_BITS[i]``: codes 0 and 1 exactly where a bf16 pair wants
  them (sign at 15 / 31, e1 e0 m at 8..6 / 24..22, which makes the pair e2m1 * 2^-126), codes 2-3 and 4-5 that
  pattern rotated left by 4 and 10 bits, codes 6-7 their mantissa bits rotated by 14 and the rest by 6 (the four
  rotations tile the 32 bits); the decode of a word into its four bf16 pairs (k, k+1) is then one mask, two
  rotate-and-masks and one two-part gather, nine integer operations (moek_common.cuh). The row's two 16-byte halves are swapped when
  bit 2 of r is set, so that 8 threads reading 16 bytes of 8 consecutive rows, or 32 lanes reading 8 bytes
  (k-group c of rows g and g + 8, the A operand of mma.sync m16n8k16), hit distinct shared-memory banks. Item rows
  0..127 are gate rows ``128t + r`` and 128..255 the matching up rows ``I + 128t + r - 128`` (gate_up), or rows
  ``256t + r`` (down).
"""
import torch

KG = 8
RUN = 16 + KG * 64  # 528: packed bytes per (expert, run of 8 k-groups, 128 positions)
# bit positions (m, e0, e1, sign) of code i of a word's 8 consecutive k
CODE_BITS = ((6, 7, 8, 15), (22, 23, 24, 31), (10, 11, 12, 19), (26, 27, 28, 3), (16, 17, 18, 25), (0, 1, 2, 9),
             (20, 13, 14, 21), (4, 29, 30, 5))


def _spread_table(device) -> torch.Tensor:
    """int64 [8, 16]: the word bits of code i with value v."""
    t = torch.zeros((8, 16), dtype=torch.int64)
    for i, bits in enumerate(CODE_BITS):
        for v in range(16):
            t[i, v] = sum(((v >> b) & 1) << pos for b, pos in enumerate(bits))
    return t.to(device)


# ------------------------------------------------------------------------------------------------------------ scales
def scale_factor(scales: torch.Tensor) -> float:
    """Power of two shared by all experts of a matrix: largest 2^j with max(nonzero) * 2^(7+j) <= 448 * 2^7."""
    v = scales.float()
    nz = v[v > 0]
    if nz.numel() == 0:
        return 1.0
    mx = float(nz.max()) * 128.0
    lim = 448.0 * 128.0
    sf = 1.0
    while mx < lim and mx * sf * 2.0 <= lim:
        sf *= 2.0
    return sf


def marlin_scale_bytes(scales: torch.Tensor, sf: float) -> torch.Tensor:
    """[E, N, K/16] float8_e4m3fn -> Marlin S0E5M3 bytes [E, K/16, N] (uint8)."""
    e, n, kg = scales.shape
    s = scales.float().transpose(1, 2).reshape(e, kg, n // 64, 8, 8)  # column 8j + i of each 64 at [.., j, i]
    s = s.transpose(-1, -2).reshape(e, kg, n)  # position 8i + j <- column i + 8j
    h = s.to(torch.float16).reshape(e, kg, n // 4, 4)[..., [0, 2, 1, 3]].reshape(e, kg, n)
    if sf > 1.0:
        h = (h.float() * sf).to(torch.float16)
    h = h * 128.0
    h = torch.where(h < 2, torch.zeros_like(h), h)
    bits = h.view(torch.int16).to(torch.int32) & 0xFFFF
    return ((bits >> 7) & 0xFF).to(torch.uint8)


def global_scale(gs: torch.Tensor, sf: float) -> torch.Tensor:
    return (gs.float() * (2.0 ** 119)) / sf


def pack_scales(s: torch.Tensor, gate_up: bool, chunk: int = 32):
    """bytes [E, K/16, N] -> (packed uint8 [E, K/128, N/128, 528], exc_off int32 [E*N/256*K/128 + 1], exc_ent int32).

    Same bytes as files/mbx_moek.py:61-120. The base of each (8 positions x 8 k-groups) block is the smallest value v
    of the block whose window [v, v + 15] holds the most values of the block.
    """
    e, kr, n = s.shape
    nb, nt = kr // KG, n // 256
    dev = s.device
    packed = torch.empty((e, nb, n // 128, RUN), dtype=torch.uint8, device=dev)
    keys, cols, kgs, vals = [], [], [], []
    for e0 in range(0, e, chunk):
        e1 = min(e, e0 + chunk)
        ec = e1 - e0
        # v[e, b, chunk, kg, p]: block (e, b, chunk) holds k-groups b*8..b*8+7 of positions chunk*8..chunk*8+7
        v = s[e0:e1].view(ec, nb, KG, n // 8, 8).permute(0, 1, 3, 2, 4).to(torch.int16)
        flat = v.reshape(ec, nb, n // 8, KG * 8)
        inwin = (flat[..., None, :] >= flat[..., :, None]) & (flat[..., None, :] <= flat[..., :, None] + 15)
        score = inwin.sum(-1).to(torch.int32) * 256 + (255 - flat.to(torch.int32))
        base = torch.gather(flat, -1, score.argmax(-1, keepdim=True))  # [ec, nb, n/8, 1]
        off = v - base[..., None]
        exc = (off < 0) | (off > 15)
        off = torch.where(exc, torch.zeros_like(off), off).to(torch.uint8)
        nib = off[..., :4] | (off[..., 4:] << 4)  # [ec, nb, n/8, KG, 4]
        body = nib.view(ec, nb, n // 128, 16, KG, 4).permute(0, 1, 2, 4, 3, 5).reshape(ec, nb, n // 128, KG * 64)
        packed[e0:e1, :, :, :16] = base.view(ec, nb, n // 128, 16).to(torch.uint8)
        packed[e0:e1, :, :, 16:] = body
        ie, ib, ic, ikg, ip = torch.nonzero(exc, as_tuple=True)
        run = ic // 16
        item = run % nt if gate_up else run // 2
        keys.append(((ie + e0) * nt + item) * nb + ib)
        cols.append(ic * 8 + ip)
        kgs.append(ikg)
        vals.append(v[ie, ib, ic, ikg, ip].to(torch.int64))
    key, col, kg, val = (torch.cat(t) for t in (keys, cols, kgs, vals))
    # entries of one (expert, item, run) list in (position chunk, k-group, position-in-chunk) order
    order = torch.argsort((key * (n // 8) + col // 8) * 64 + kg * 8 + col % 8)
    key, col, kg, val = key[order], col[order], kg[order], val[order]
    cnt = torch.bincount(key, minlength=e * nt * nb)
    exc_off = torch.zeros(e * nt * nb + 1, dtype=torch.int32, device=dev)
    exc_off[1:] = torch.cumsum(cnt, 0).to(torch.int32)
    word = col | (kg << 16) | (val << 24)
    word = torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)
    ent = word if word.numel() else torch.zeros(1, dtype=torch.int32, device=dev)
    return packed, exc_off, ent


def tile_scales(packed: torch.Tensor, n: int, gate_up: bool) -> torch.Tensor:
    """[E, nb, N/128, 528] -> [E, N/256, nb, 1056]: an item's two runs side by side (files/mbx_moek.py:163-172)."""
    e, nb = packed.shape[:2]
    nt = n // 256
    t = torch.arange(nt, device=packed.device)
    runs = torch.stack([t, nt + t], 1) if gate_up else torch.stack([2 * t, 2 * t + 1], 1)
    return packed[:, :, runs.flatten(), :].view(e, nb, nt, 2 * RUN).transpose(1, 2).contiguous()


# ----------------------------------------------------------------------------------------------------------- weights
def item_columns(n: int, gate_up: bool, device=None) -> torch.Tensor:
    """Logical column of every item slot: [N/256, 256]."""
    nt = n // 256
    slot = torch.arange(256, device=device)
    t = torch.arange(nt, device=device)[:, None]
    if gate_up:
        return torch.where(slot < 128, 128 * t + slot, n // 2 + 128 * t + slot - 128)
    return 256 * t + slot


def _swizzle_rows(device) -> torch.Tensor:
    """Rows of a stage block whose two 16-byte halves are swapped (bit 2 of the row index set)."""
    return ((torch.arange(256, device=device) >> 2) & 1).bool()


def tile_weights(codes: torch.Tensor, gate_up: bool, chunk: int = 16) -> torch.Tensor:
    """Checkpoint codes uint8 [E, N, K/2] -> this build's tiled int32 [E, K/16, 2N] (see the module docstring)."""
    e, n, k2 = codes.shape
    k = 2 * k2
    nt, ns = n // 256, k // 64
    cols = item_columns(n, gate_up, codes.device).flatten()
    spread = _spread_table(codes.device)
    slot_i = torch.arange(8, device=codes.device)
    swap = _swizzle_rows(codes.device)
    out = torch.empty((e, k // 16, 2 * n), dtype=torch.int32, device=codes.device)
    for e0 in range(0, e, chunk):
        e1 = min(e, e0 + chunk)
        c = codes[e0:e1][:, cols, :]
        nib = torch.stack([c & 0xF, c >> 4], -1).view(e1 - e0, nt, 256, ns, 8, 8)  # [e, t, r, s, w, i]
        word = spread[slot_i, nib.permute(0, 1, 3, 2, 4, 5).long()].sum(-1)  # [e, t, s, r, w]
        word = word.view(e1 - e0, nt, ns, 256, 2, 4)
        word[:, :, :, swap] = word[:, :, :, swap].flip(-2)
        word = torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)
        out[e0:e1] = word.reshape(e1 - e0, k // 16, 2 * n)
    return out


def untile_weights(w: torch.Tensor, n: int, gate_up: bool) -> torch.Tensor:
    """Inverse of ``tile_weights``: int32 [E, K/16, 2N] -> checkpoint codes uint8 [E, N, K/2]."""
    e = w.shape[0]
    k = w.shape[1] * 16
    nt, ns = n // 256, k // 64
    pos = torch.tensor(CODE_BITS, dtype=torch.int64, device=w.device)  # [8 codes, 4 bits]
    word = (w.to(torch.int64) & 0xFFFFFFFF).view(e, nt, ns, 256, 2, 4).clone()
    swap = _swizzle_rows(w.device)
    word[:, :, :, swap] = word[:, :, :, swap].flip(-2)
    bits = (word.view(e, nt, ns, 256, 8)[..., None, None] >> pos) & 1  # [e, t, s, r, w, i, b]
    nib = (bits << torch.arange(4, device=w.device)).sum(-1).to(torch.uint8)  # [e, t, s, r, w, i]
    nib = nib.permute(0, 1, 3, 2, 4, 5).reshape(e, nt * 256, k)
    out = torch.empty((e, n, k), dtype=torch.uint8, device=w.device)
    out[:, item_columns(n, gate_up, w.device).flatten(), :] = nib
    return (out[..., 0::2] | (out[..., 1::2] << 4)).contiguous()


# ------------------------------------------------------------------------------------------------------------- layer
class PreparedMatrix:
    """One matrix of a layer in the kernels' format. On a CUDA device the conversion runs in this build's prep
    kernels (``native``, csrc/moek_prep.cu); elsewhere, or with ``native=False``, in the torch restatement above
    (the same bytes: tests/test_gpu_prep.py compares the two)."""

    def __init__(self, codes, scales, gs, gate_up: bool, native=None):
        e, n, k2 = codes.shape
        k = 2 * k2
        check_shapes(n, k, gate_up)
        self.gate_up, self.E, self.N, self.K = gate_up, e, n, k
        if native is None:
            native = codes.is_cuda
        if native:
            self._prepare_native(codes, scales, gs)
            return
        self.sf = scale_factor(scales)
        sb = marlin_scale_bytes(scales, self.sf)
        packed, self.exc_off, self.exc_ent = pack_scales(sb, gate_up)
        self.sp = tile_scales(packed, n, gate_up)
        self.g = global_scale(gs, self.sf).contiguous()
        self.w = tile_weights(codes, gate_up)

    def _prepare_native(self, codes, scales, gs):
        import ctypes

        from ._lib import call

        e, n, k, gu = self.E, self.N, self.K, int(self.gate_up)
        dev = codes.device
        codes = codes.contiguous()
        sc = scales.contiguous().view(torch.uint8)
        gs = gs.float().contiguous()
        st = torch.cuda.current_stream(dev).cuda_stream
        wsb = ctypes.c_size_t(0)
        call("moek_prep_workspace_bytes", e, n, k, ctypes.byref(wsb))
        ws = torch.empty(wsb.value, dtype=torch.uint8, device=dev)
        nkeys = e * (n // 256) * (k // 128)
        self.sp = torch.empty((e, n // 256, k // 128, 2 * RUN), dtype=torch.uint8, device=dev)
        self.g = torch.empty(e, dtype=torch.float32, device=dev)
        self.exc_off = torch.empty(nkeys + 1, dtype=torch.int32, device=dev)
        sf, nexc = ctypes.c_float(0.0), ctypes.c_int64(0)
        call("moek_prep_scales", sc.data_ptr(), gs.data_ptr(), e, n, k, gu, ws.data_ptr(), ws.numel(),
             self.sp.data_ptr(), self.g.data_ptr(), self.exc_off.data_ptr(), ctypes.byref(sf), ctypes.byref(nexc), st)
        self.sf = float(sf.value)
        self.exc_ent = torch.zeros(max(1, nexc.value), dtype=torch.int32, device=dev)
        if nexc.value:
            call("moek_prep_exceptions", sc.data_ptr(), e, n, k, gu, sf, ws.data_ptr(), self.exc_off.data_ptr(),
                 self.exc_ent.data_ptr(), st)
        self.w = torch.empty((e, k // 16, 2 * n), dtype=torch.int32, device=dev)
        call("moek_prep_weights", codes.data_ptr(), e, n, k, gu, self.w.data_ptr(), st)

    def nbytes(self) -> int:
        """Bytes the kernels read for the whole matrix (weights + packed scales + exception lists)."""
        return (self.w.numel() * 4 + self.sp.numel() + self.exc_off.numel() * 4
                + int(self.exc_off[-1]) * 4)


def check_shapes(n: int, k: int, gate_up: bool):
    if k % 128 or n % 256 or (gate_up and (n // 2) % 128):
        raise ValueError(f"moek_b200: unsupported matrix N={n}, K={k} (need K % 128 == 0, N % 256 == 0"
                         + (", N/2 % 128 == 0)" if gate_up else ")"))


class PreparedLayer:
    """Both matrices of one routed-expert layer (w13 = gate rows then up rows, w2 = down)."""

    def __init__(self, w13, w2, native=None):
        self.w13 = PreparedMatrix(*w13, gate_up=True, native=native)
        self.w2 = PreparedMatrix(*w2, gate_up=False, native=native)
        self.E = self.w13.E
        self.hidden = self.w13.K
        self.inter = self.w13.N // 2
        if self.w2.N != self.hidden or self.w2.K != self.inter or self.w2.E != self.E:
            raise ValueError("moek_b200: w13 and w2 shapes do not belong to one layer")

    def expert_bytes(self) -> torch.Tensor:
        """Per-expert bytes both matrices stream when the expert is touched: [E] int64 (weights + packed scales +
        that expert's exception entries and offsets)."""
        out = []
        for m in (self.w13, self.w2):
            per = m.w[0].numel() * 4 + m.sp[0].numel()
            nkeys = (m.exc_off.numel() - 1) // m.E
            off = m.exc_off.to(torch.int64)
            n_exc = off[nkeys::nkeys][:m.E] - off[0:-1:nkeys][:m.E]
            out.append(per + 4 * n_exc + 4 * (nkeys + 1))
        return out[0] + out[1]
