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
