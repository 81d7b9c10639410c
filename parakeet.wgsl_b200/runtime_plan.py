"""Weight-format contract of the parakeet.wgsl packages (host side, numpy).

Restates the pieces of ``src/model/runtime-plan.ts`` and ``model/convert.py``
that define how the encoder's weights are laid out, so packages produced for
the reference load here unchanged:

* layout strings (runtime-plan.ts:26-37) and ``palette_bits_for_layout``
  (runtime-plan.ts:352-368);
* LSB-first palette code packing, 32 five-bit or 16 six-bit codes per group of
  5 / 3 little-endian u32 words, in k-by-output row-major (K-major) order
  (convert.py:2130-2157) -- ``pack_codes`` / ``unpack_codes``;
* palette validation (``validatePalettePair``, runtime-plan.ts:529-588);
* the n256/n128-k32 tile-major index map (runtime-plan.ts:454-490);
* the Transformer-XL relative-position table, its f32 projection and the
  head-vector-position-vec4 packing (convert.py:1143-1228).
"""
from __future__ import annotations

import math

import numpy as np

RUNTIME_STORAGE_ALIGNMENT = 256
ROW_MAJOR_F16_LAYOUT = "k-by-output-row-major-f16"
TILE_MAJOR_F16_LAYOUT = "n256-k32-tile-major-f16"
ROW_MAJOR_F32_LAYOUT = "k-by-output-row-major-f32"
TILE_MAJOR_F32_LAYOUT = "n128-k32-tile-major-f32"
PALETTE5_LAYOUT = "k-by-output-row-major-palette5-lsb-u32"
PALETTE6_LAYOUT = "k-by-output-row-major-palette6-lsb-u32"
PALETTE_LUT_LAYOUT = "output-group-by-palette-lut"
TILE_INNER = 32


def palette_bits_for_layout(layout: str) -> int | None:
    return {PALETTE5_LAYOUT: 5, PALETTE6_LAYOUT: 6}.get(layout)


def palette_layout(bits: int) -> str:
    return {5: PALETTE5_LAYOUT, 6: PALETTE6_LAYOUT}[bits]


def code_group(bits: int) -> tuple[int, int]:
    """(codes per group, u32 words per group)."""
    if bits == 5:
        return 32, 5
    if bits == 6:
        return 16, 3
    raise ValueError(f"Unsupported palette code width {bits}")


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack unsigned codes LSB-first into [groups, words] little-endian u32."""
    per, words = code_group(bits)
    flat = np.ascontiguousarray(codes).reshape(-1)
    if flat.size % per:
        raise ValueError(f"{bits}-bit palette code count {flat.size} is not divisible by {per}")
    if flat.size and (int(flat.min()) < 0 or int(flat.max()) >= 1 << bits):
        raise ValueError(f"{bits}-bit palette codes must be in [0, {1 << bits})")
    grouped = flat.astype(np.uint64).reshape(-1, per)
    out = np.zeros((grouped.shape[0], words), dtype="<u4")
    for i in range(per):
        bit = i * bits
        w, s = bit // 32, bit % 32
        out[:, w] |= ((grouped[:, i] << np.uint64(s)) & np.uint64(0xFFFFFFFF)).astype("<u4")
        if s + bits > 32:
            out[:, w + 1] |= (grouped[:, i] >> np.uint64(32 - s)).astype("<u4")
    return out


def unpack_codes(packed: np.ndarray, bits: int) -> np.ndarray:
    """Inverse of ``pack_codes``: one uint8 code per scalar."""
    per, words = code_group(bits)
    p = np.ascontiguousarray(packed, dtype="<u4").reshape(-1, words).astype(np.uint64)
    out = np.empty((p.shape[0], per), dtype=np.uint8)
    mask = np.uint64((1 << bits) - 1)
    for i in range(per):
        bit = i * bits
        w, s = bit // 32, bit % 32
        v = p[:, w] >> np.uint64(s)
        if s + bits > 32:
            v |= p[:, w + 1] << np.uint64(32 - s)
        out[:, i] = (v & mask).astype(np.uint8)
    return out.reshape(-1)


def validate_palette_pair(inner: int, columns: int, packed: np.ndarray, palette: np.ndarray, bits: int) -> int:
    """validatePalettePair: returns the palette group width (columns / G)."""
    per, words = code_group(bits)
    if columns % per or (inner * columns) % per:
        raise ValueError("palette codes are not group aligned")
    if tuple(packed.shape) != (inner * columns // per, words):
        raise ValueError("invalid packed palette storage")
    if palette.ndim != 2 or palette.shape[1] != 1 << bits:
        raise ValueError("invalid palette storage")
    groups = palette.shape[0]
    if columns % groups or (columns // groups) % per:
        raise ValueError("palette does not partition output columns")
    return columns // groups


def expand(packed: np.ndarray, palette: np.ndarray, bits: int, inner: int, columns: int) -> np.ndarray:
    """Dense [K, N] weight from packed codes (host-side helper for packaging)."""
    group_cols = validate_palette_pair(inner, columns, packed, palette, bits)
    codes = unpack_codes(packed, bits).reshape(inner, columns).astype(np.int64)
    pg = np.minimum(np.arange(columns) // group_cols, palette.shape[0] - 1)
    return palette[pg[None, :], codes]


def tile_major_index(scalar: int, inner: int, columns: int, tile_cols: int) -> int:
    """runtimeGemmTileMajorScalarIndexForColumns (runtime-plan.ts:454-490)."""
    if inner % TILE_INNER or columns % tile_cols:
        raise ValueError(f"Tile-major runtime weights require K%32=0 and N%{tile_cols}=0")
    if not 0 <= scalar < inner * columns:
        raise ValueError("Tile-major scalar index exceeds the logical KxN matrix")
    k, n = divmod(scalar, columns)
    return ((n // tile_cols * (inner // TILE_INNER) + k // TILE_INNER) * TILE_INNER + k % TILE_INNER) * tile_cols \
        + n % tile_cols


def build_relative_positions(encoder_frames: int = 188, channels: int = 1024) -> np.ndarray:
    """Descending Transformer-XL sin/cos table [2T-1, C] in f32."""
    positions = np.arange(encoder_frames - 1, -encoder_frames, -1, dtype=np.float32).reshape(-1, 1)
    channel_indices = np.arange(0, channels, 2, dtype=np.float32)
    exponent = np.float32(-(math.log(10_000.0) / channels))
    div_term = np.exp(channel_indices * exponent)
    angles = positions * div_term.reshape(1, -1)
    table = np.empty((2 * encoder_frames - 1, channels), dtype=np.float32)
    table[:, 0::2] = np.sin(angles)
    table[:, 1::2] = np.cos(angles)
    return table


def project_relative_positions(table: np.ndarray, weight_out_in: np.ndarray, dtype=np.float16) -> np.ndarray:
    """nn.Linear orientation: table @ W^T in f32, cast to the package dtype."""
    projected = np.asarray(table, dtype=np.float32) @ np.asarray(weight_out_in, dtype=np.float32).T
    return np.ascontiguousarray(projected, dtype=dtype)


def pack_projected_relative_positions(projected: np.ndarray, heads: int = 8, vector_width: int = 4) -> np.ndarray:
    """[P, C] -> head-vector-position-vec4 [heads, head/4, P, 4]."""
    p_rows, channels = projected.shape
    head = channels // heads
    return np.ascontiguousarray(
        projected.reshape(p_rows, heads, head // vector_width, vector_width).transpose(1, 2, 0, 3))
