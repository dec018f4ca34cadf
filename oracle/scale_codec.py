"""The kit's lossless packed-scale codec and its item tiling, restated in numpy (test infrastructure only).

Follows files/mbx_moek.py:61-137 (``pack_scales``, ``pack_scales_part``, ``unpack_scales``) and :163-172
(``tile_scales``). Input: Marlin S0E5M3 scale bytes [E, K/16, N] (``oracle.marlin_scales``).

Format, per (expert e, run b of KG=8 consecutive k-groups, 128 positions): 16 base bytes (one per 8 positions) then
KG rows of 64 bytes of 4-bit offsets; byte i of an 8-position chunk holds position i in its low nibble and position
i + 4 in its high nibble. The base of a chunk's 64 scales (8 positions x KG k-groups) is the start of the 16-value
window that covers most of them (smallest such start on ties). Scales outside the window store offset 0 and an
int32 exception entry ``position | kg << 16 | value << 24`` in a list per (expert, item, run); ``item`` is the
kernel's 256-column tile (gate_up: gate run r pairs with up run N/256 + r; down: runs 2r and 2r + 1).
``exc_off`` holds the prefix sums of the list lengths in (expert, item, run) order.
"""
import numpy as np

KG = 8
RUN = 16 + KG * 64  # 528 bytes per (expert, run, 128 positions)


def pack_scales(s: np.ndarray, gate_up: bool):
    """bytes [E, K/16, N] -> (packed uint8 [E, K/128, N/128, 528], exc_off int32, exc_ent int32)."""
    e, kr, n = s.shape
    nb, nt = kr // KG, n // 256
    packed = np.zeros((e, nb, n // 128, RUN), dtype=np.uint8)
    lists = {}
    for ei in range(e):
        for b in range(nb):
            blk = s[ei, b * KG:(b + 1) * KG, :].astype(np.int32)  # [KG, n]
            # v[chunk, kg * 8 + p] (files/mbx_moek.py:92)
            v = blk.reshape(KG, n // 8, 8).transpose(1, 0, 2).reshape(n // 8, KG * 8)
            srt = np.sort(v, axis=1)
            hi = np.stack([np.searchsorted(row, row + 15, side="right") for row in srt])
            cover = hi - np.arange(KG * 8)[None, :]
            base = srt[np.arange(n // 8), cover.argmax(1)]  # first maximum
            off = v - base[:, None]
            exc = (off < 0) | (off > 15)
            off = np.where(exc, 0, off).astype(np.uint8).reshape(n // 8, KG, 8)
            nib = off[:, :, :4] | (off[:, :, 4:] << 4)  # [n/8, KG, 4]
            for r in range(n // 128):
                packed[ei, b, r, :16] = base[r * 16:(r + 1) * 16]
                body = nib[r * 16:(r + 1) * 16].transpose(1, 0, 2).reshape(KG, 64)
                packed[ei, b, r, 16:] = body.reshape(-1)
            for chunk, i in zip(*np.nonzero(exc)):
                run = chunk // 16
                item = run % nt if gate_up else run // 2
                key = (ei * nt + item) * nb + b
                col, kg = chunk * 8 + i % 8, i // 8
                word = int(col) | (int(kg) << 16) | (int(v[chunk, i]) << 24)
                lists.setdefault(key, []).append(word - (1 << 32) if word >= 1 << 31 else word)
    nkeys = e * nt * nb
    exc_off = np.zeros(nkeys + 1, dtype=np.int32)
    ent = []
    for key in range(nkeys):
        lst = lists.get(key, [])
        ent.extend(lst)
        exc_off[key + 1] = exc_off[key] + len(lst)
    exc_ent = np.array(ent if ent else [0], dtype=np.int32)
    return packed, exc_off, exc_ent


def unpack_scales(packed: np.ndarray, exc_off: np.ndarray, ent: np.ndarray, kr: int, n: int,
                  gate_up: bool) -> np.ndarray:
    """Inverse of ``pack_scales`` on the untiled layout -> bytes [E, K/16, N] (files/mbx_moek.py:123-137)."""
    e, nb = packed.shape[:2]
    nt = n // 256
    out = np.zeros((e, kr, n), dtype=np.uint8)
    for ei in range(e):
        for b in range(nb):
            for r in range(n // 128):
                run = packed[ei, b, r]
                base = run[:16].astype(np.int32)
                body = run[16:].reshape(KG, 16, 4)
                for kg in range(KG):
                    lo, hi = body[kg] & 0xF, body[kg] >> 4  # [16 chunks, 4]
                    vals = np.concatenate([lo, hi], 1).astype(np.int32) + base[:, None]
                    out[ei, b * KG + kg, r * 128:(r + 1) * 128] = vals.reshape(-1)
    for key in range(e * nt * nb):
        ei, b = key // (nt * nb), key % nb
        for w in ent[exc_off[key]:exc_off[key + 1]]:
            w = int(w) & 0xFFFFFFFF
            col, kg, val = w & 0xFFFF, (w >> 16) & 0xFF, (w >> 24) & 0xFF
            out[ei, b * KG + kg, col] = val
    return out


def tile_scales(packed: np.ndarray, n: int, gate_up: bool) -> np.ndarray:
    """packed [E, nb, N/128, 528] -> per (expert, item, run) the item's two runs: [E, N/256, nb, 1056]."""
    e, nb = packed.shape[:2]
    nt = n // 256
    out = np.zeros((e, nt, nb, 2 * RUN), dtype=np.uint8)
    for t in range(nt):
        r0, r1 = (t, nt + t) if gate_up else (2 * t, 2 * t + 1)
        out[:, t, :, :RUN] = packed[:, :, r0]
        out[:, t, :, RUN:] = packed[:, :, r1]
    return out
