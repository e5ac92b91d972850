"""Sort-key width policy of sort_and_bin (splax/_rasterize/_sort/_sort.py:23-66).

The kernels take the key width as an explicit argument; this module decides it in Python so
that tests can monkeypatch ``_use_32bit_keys`` exactly as the reference's tests do
(tests/test_warp_batch.py:45-56, tests/test_warp_rasterize.py:250-260).
"""

from __future__ import annotations

BLOCK_WIDTH = 16


def _use_32bit_keys(depth_bits: int) -> bool:
    # The packed key needs at least 16 depth bits below the image and tile ids.
    return depth_bits >= 16


def key_fields(B: int, img_h: int, img_w: int) -> tuple[int, int, int]:
    """(tile_n_bits, image_n_bits, depth_bits) of the packed key for B images of H x W."""
    num_tiles = ((img_w + BLOCK_WIDTH - 1) // BLOCK_WIDTH) * ((img_h + BLOCK_WIDTH - 1) // BLOCK_WIDTH)
    tile_n_bits = (num_tiles - 1).bit_length()
    image_n_bits = (B - 1).bit_length()
    return tile_n_bits, image_n_bits, 31 - image_n_bits - tile_n_bits


def key_bits_for(B: int, img_h: int, img_w: int) -> int:
    """32 for the packed key, 64 for the wide one; raises ValueError on key overflow."""
    tile_n_bits, image_n_bits, depth_bits = key_fields(B, img_h, img_w)
    if _use_32bit_keys(depth_bits):
        return 32
    upper = image_n_bits + tile_n_bits
    if upper > 32:
        raise ValueError(
            f"batched intersection key overflow: image_n_bits({image_n_bits}) + "
            f"tile_n_bits({tile_n_bits}) = {upper} > 32 "
            f"(batch B={B}, n_tiles={(1 << tile_n_bits)}). Reduce batch size or resolution.")
    return 64
