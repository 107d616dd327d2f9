"""GGML block formats handled by the B200 expert path.

Type ids and block geometry are those of the reference's dispatcher
(``cpp/dequant_k.cpp:37-41`` and ``:302-322``) and of ``SUPPORTED_TYPES``
(``src/flash_moe/native_expert.py:10``).
"""
from __future__ import annotations

Q8_0 = 8
Q3_K = 11
Q4_K = 12
Q5_K = 13
Q6_K = 14

SUPPORTED_TYPES = frozenset({Q8_0, Q3_K, Q4_K, Q5_K, Q6_K})

# type id -> (values per block, bytes per block)
BLOCK: dict[int, tuple[int, int]] = {
    Q8_0: (32, 34),
    Q3_K: (256, 110),
    Q4_K: (256, 144),
    Q5_K: (256, 176),
    Q6_K: (256, 210),
}

NAMES = {Q8_0: "Q8_0", Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}


def block_size(type_id: int) -> int:
    return BLOCK.get(int(type_id), (0, 0))[0]


def block_bytes(type_id: int) -> int:
    return BLOCK.get(int(type_id), (0, 0))[1]


def row_bytes(type_id: int, columns: int) -> int:
    """Bytes of one row of ``columns`` values; raises if not block aligned."""
    bs, pb = BLOCK[int(type_id)]
    if columns % bs:
        raise ValueError(f"{columns} columns is not a multiple of the "
                         f"{NAMES[int(type_id)]} block size {bs}")
    return columns // bs * pb


def tensor_bytes(type_id: int, rows: int, columns: int) -> int:
    return rows * row_bytes(type_id, columns)
