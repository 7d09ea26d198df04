"""MXFP8 (OCP microscaling, e4m3 elements + e8m0 power-of-two scale per 32 elements).

PyTorch reference of the exact quantization the sm_100a kernels perform, plus the
scale-factor *atom* layout the tcgen05 block-scaled GEMM consumes.

Scale rule (same as the reference's RMSNorm+MXFP8 quantizer,
worker/zstep_worker/kernels_sm120/norm_quant.py:63-67): for a 32-element block with
absolute maximum ``amax`` the scale is ``2**e`` with ``e = ceil(log2(amax / 448))``
clamped to [-127, 127]; elements are ``e4m3(x / 2**e)`` (round to nearest even).  An
all-zero block gets code 0.

Atom layout: scale codes of a ``[rows, k]`` matrix are stored as
``[ceil(rows/128), k/128, 512]`` bytes; inside an atom, row ``r = r0 + 32*r1`` and
32-wide block ``j`` (of the atom's 4) live at byte ``r0*16 + r1*4 + j``.
"""

from __future__ import annotations

import torch

E4M3_MAX = 448.0


def e8m0_codes(amax: torch.Tensor) -> torch.Tensor:
    """Exact ``clamp(ceil(log2(amax/448)), -127, 127) + 127`` as uint8 (0 for amax == 0)."""
    r = amax.float() / E4M3_MAX
    mant, exp = torch.frexp(r)  # r = mant * 2**exp, mant in [0.5, 1)
    e = torch.where(mant == 0.5, exp - 1, exp)
    e = e.clamp(-127, 127)
    code = (e + 127).to(torch.int32)
    code = torch.where(amax > 0, code, torch.zeros_like(code))
    return code.to(torch.uint8)


def code_to_scale(code: torch.Tensor) -> torch.Tensor:
    c = code.to(torch.int32)
    return torch.where(c == 0, torch.full_like(c, 0, dtype=torch.float32) + 2.0**-127,
                       torch.pow(2.0, (c - 127).float()))


def quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize ``x [rows, k]`` (k % 32 == 0) -> (e4m3 bytes uint8 [rows, k], codes uint8 [rows, k/32])."""
    rows, k = x.shape
    assert k % 32 == 0
    xb = x.float().reshape(rows, k // 32, 32)
    amax = xb.abs().amax(dim=-1)
    code = e8m0_codes(amax)
    c = code.to(torch.int32)
    inv = torch.pow(2.0, (127 - c).float())
    inv = torch.where(c == 0, torch.pow(torch.tensor(2.0, device=x.device), 127.0), inv)
    scaled = (xb * inv.unsqueeze(-1)).clamp(-E4M3_MAX, E4M3_MAX)
    q = scaled.to(torch.float8_e4m3fn).view(torch.uint8).reshape(rows, k)
    return q, code


def dequantize(q: torch.Tensor, code: torch.Tensor) -> torch.Tensor:
    rows, k = q.shape
    vals = q.view(torch.float8_e4m3fn).float().reshape(rows, k // 32, 32)
    return (vals * code_to_scale(code).unsqueeze(-1)).reshape(rows, k)


def atoms_from_codes(code: torch.Tensor) -> torch.Tensor:
    """[rows, k/32] codes -> flat atom buffer [ceil(rows/128) * (k/128) * 512] uint8."""
    rows, nkb = code.shape
    assert nkb % 4 == 0
    rb = (rows + 127) // 128
    padded = torch.zeros(rb * 128, nkb, dtype=torch.uint8, device=code.device)
    padded[:rows] = code
    # [rb, r1(4), r0(32), kt, j(4)] -> [rb, kt, r0, r1, j]
    t = padded.reshape(rb, 4, 32, nkb // 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return t.reshape(-1)


def codes_from_atoms(atoms: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    nkb = k // 32
    rb = (rows + 127) // 128
    t = atoms[: rb * (nkb // 4) * 512].reshape(rb, nkb // 4, 32, 4, 4).permute(0, 3, 2, 1, 4)
    return t.reshape(rb * 128, nkb)[:rows].contiguous()


def atoms_bytes(rows: int, k: int) -> int:
    return ((rows + 127) // 128) * (k // 128) * 512


def quantize_to_atoms(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    q, code = quantize(x)
    return q, atoms_from_codes(code)


def tile_weight(q: torch.Tensor) -> torch.Tensor:
    """Row-major e4m3 weight [rows, k] (rows % 128 == 0, k % 128 == 0) -> the GEMM's
    pre-tiled, pre-swizzled layout: every 128x128-byte block of one (feature tile,
    K tile) becomes one contiguous 16 KiB chunk ([rows/128][k/128][128][128]) whose
    16-byte pieces are already in the 128-byte-swizzle order (piece c of row r stored
    at piece c ^ (r % 8)).  A plain bulk copy of the chunk to a 1024-byte aligned
    shared-memory buffer then yields exactly the image a swizzled TMA load would."""
    rows, k = q.shape
    t = q.view(rows // 128, 128, k // 128, 128).permute(0, 2, 1, 3)  # [mt, kt, 128 r, 128 B]
    t = t.reshape(rows // 128, k // 128, 16, 8, 8, 16)              # [.., row grp, r%8, piece, 16 B]
    j = torch.arange(8, device=q.device)
    src_piece = (j[None, :] ^ j[:, None])                           # [r%8, dst piece] -> src piece
    idx = src_piece.view(1, 1, 1, 8, 8, 1).expand(t.shape)
    t = torch.gather(t, 4, idx)
    return t.contiguous().view(rows, k)


def fake_quant(x: torch.Tensor) -> torch.Tensor:
    """Quantize-dequantize round trip (the value an MXFP8 GEMM actually multiplies)."""
    q, code = quantize(x)
    return dequantize(q, code).to(x.dtype) if x.dtype != torch.float32 else dequantize(q, code)


# ------------------------------------------------------------------------------ MXFP4
# OCP MXFP4: e2m1 elements (sign, 2 exponent bits with bias 1, 1 mantissa bit; magnitudes
# 0, 0.5, 1, 1.5, 2, 3, 4, 6) with the same e8m0 scale per 32 elements.  The scale is
# ``2**ceil(log2(amax / 6))``; elements round to the nearest e2m1 value, ties to the even
# mantissa.  Two elements per byte: element 2i in the low nibble, 2i+1 in the high one.
# Every e2m1 value times an e8m0 scale is exactly an e4m3 value times the same scale, so
# the GEMM widens MXFP4 weights to MXFP8 in shared memory without changing a product.

E2M1_MAX = 6.0
E2M1_MAGS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def e8m0_codes_fp4(amax: torch.Tensor) -> torch.Tensor:
    r = amax.float() / E2M1_MAX
    mant, exp = torch.frexp(r)
    e = torch.where(mant == 0.5, exp - 1, exp).clamp(-127, 127)
    code = (e + 127).to(torch.int32)
    return torch.where(amax > 0, code, torch.zeros_like(code)).to(torch.uint8)


# Rounding boundaries between consecutive e2m1 magnitudes; at an exact boundary the
# value goes to the neighbour with the even mantissa (the upper one after odd boundaries).
_E2M1_BOUNDS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


def quantize_fp4(x: torch.Tensor, chunk_rows: int = 4096) -> tuple[torch.Tensor, torch.Tensor]:
    """``x [rows, k]`` (k % 32 == 0) -> (packed e2m1 uint8 [rows, k/2], codes uint8 [rows, k/32])."""
    rows, k = x.shape
    assert k % 32 == 0
    packed = torch.empty(rows, k // 2, dtype=torch.uint8, device=x.device)
    codes = torch.empty(rows, k // 32, dtype=torch.uint8, device=x.device)
    for r0 in range(0, rows, chunk_rows):
        xb = x[r0:r0 + chunk_rows].float().reshape(-1, k // 32, 32)
        code = e8m0_codes_fp4(xb.abs().amax(dim=-1))
        c = code.to(torch.int32)
        inv = torch.where(c == 0, torch.full_like(c, 0, dtype=torch.float32) + 2.0 ** 127,
                          torch.pow(2.0, (127 - c).float()))
        y = (xb * inv.unsqueeze(-1)).clamp(-E2M1_MAX, E2M1_MAX)
        a = y.abs()
        mag = torch.zeros(a.shape, dtype=torch.uint8, device=x.device)
        for i, b in enumerate(_E2M1_BOUNDS):
            mag += (a > b) | ((a == b) & (i % 2 == 1))
        nib = (mag | ((y < 0).to(torch.uint8) << 3)).reshape(-1, k)
        packed[r0:r0 + chunk_rows] = nib[:, 0::2] | (nib[:, 1::2] << 4)
        codes[r0:r0 + chunk_rows] = code
    return packed, codes


def dequantize_fp4(packed: torch.Tensor, code: torch.Tensor) -> torch.Tensor:
    rows = packed.shape[0]
    k = packed.shape[1] * 2
    nib = torch.stack([packed & 0xF, packed >> 4], dim=-1).reshape(rows, k).long()
    mags = torch.tensor(E2M1_MAGS, device=packed.device)
    v = mags[nib & 7] * torch.where((nib & 8) != 0, -1.0, 1.0)
    return (v.reshape(rows, k // 32, 32) * code_to_scale(code).unsqueeze(-1)).reshape(rows, k)


def fake_quant_fp4(x: torch.Tensor) -> torch.Tensor:
    p, c = quantize_fp4(x.reshape(-1, x.shape[-1]))
    return dequantize_fp4(p, c).reshape(x.shape).to(x.dtype)


def fp4_to_e4m3(packed: torch.Tensor) -> torch.Tensor:
    """Widen packed e2m1 [rows, k/2] to e4m3 bytes [rows, k] (exact; same scales)."""
    rows = packed.shape[0]
    nib = torch.stack([packed & 0xF, packed >> 4], dim=-1).reshape(rows, -1).long()
    mags = torch.tensor(E2M1_MAGS, device=packed.device)
    v = mags[nib & 7] * torch.where((nib & 8) != 0, -1.0, 1.0)
    return v.to(torch.float8_e4m3fn).view(torch.uint8)


def tile_weight_fp4(packed: torch.Tensor) -> torch.Tensor:
    """Packed e2m1 weight [rows, k/2] (rows % 128 == 0, k % 128 == 0) -> contiguous 8 KiB
    chunks [rows/128][k/128][128 rows][64 bytes], one per (feature tile, K tile), in plain
    row-major order; the GEMM's converter warps apply the 128-byte swizzle when they widen
    a chunk to e4m3 in shared memory."""
    rows, kh = packed.shape
    t = packed.view(rows // 128, 128, kh // 64, 64).permute(0, 2, 1, 3)
    return t.contiguous().view(rows, kh)
