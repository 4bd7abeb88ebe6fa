"""GGUF tensor types on the dequant + matmul path: ids, block geometry, sizes.

This table replaces the reference loader's type mapping, which has no entries
for Q4_K (id 12) or Q6_K (id 14) and sizes Q8_0 at 36 bytes per 32 weights
instead of 34 (nodestor/crates/nodestor-formats/src/gguf.rs:268-304;
nodestor/crates/nodestor-core/src/types.rs:244-300).  The ids are ggml's
(`ggml_type`), so a GGUF tensor-info record maps straight onto them.
"""
from __future__ import annotations

from dataclasses import dataclass

Q4_0 = 2
Q8_0 = 8
Q4_K = 12
Q5_K = 13
Q6_K = 14

# Q6_K / Q5_K byte layouts.  GGML is what llama.cpp writes; NODESTOR is the
# element mapping of the reference's own code (Q6_K: nodestor/crates/
# nodestor-vulkan/shaders/dequant_q6k.comp:50-99; Q5_K: the high-bit mapping
# of nodestor/crates/nodestor-inference/src/dequant/q5_k.rs:57-70): same
# field offsets, different unpacking.
Q6K_GGML = 0
Q6K_NODESTOR = 1


@dataclass(frozen=True)
class BlockFormat:
    name: str
    type_id: int
    block_weights: int  # weights per (super-)block, along K
    block_bytes: int    # bytes per (super-)block

    def row_bytes(self, k: int) -> int:
        if k % self.block_weights:
            raise ValueError(f"{self.name}: K={k} is not a multiple of {self.block_weights}")
        return (k // self.block_weights) * self.block_bytes

    def tensor_bytes(self, n: int, k: int) -> int:
        return n * self.row_bytes(k)


FORMATS = {
    Q4_0: BlockFormat("Q4_0", Q4_0, 32, 18),
    Q8_0: BlockFormat("Q8_0", Q8_0, 32, 34),
    Q4_K: BlockFormat("Q4_K", Q4_K, 256, 144),
    Q5_K: BlockFormat("Q5_K", Q5_K, 256, 176),
    Q6_K: BlockFormat("Q6_K", Q6_K, 256, 210),
}

BY_NAME = {f.name: f for f in FORMATS.values()}


def fmt(type_id_or_name) -> BlockFormat:
    if isinstance(type_id_or_name, str):
        return BY_NAME[type_id_or_name.upper()]
    return FORMATS[int(type_id_or_name)]


def weight_bytes_per_element(type_id: int) -> float:
    f = FORMATS[type_id]
    return f.block_bytes / f.block_weights
