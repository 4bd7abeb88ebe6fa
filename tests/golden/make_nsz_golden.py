"""Generate tests/golden/nsz_golden.npz from the reference's own NSZ file.

Run from the repository root, with the path of the reference's file:
    python tests/golden/make_nsz_golden.py <reference root>/nodestor/micro_modelo_ignition.nsz

Source of truth: nodestor/micro_modelo_ignition.nsz, written by the
reference's converter (nodestor-cli/src/bin/nsz_convert.rs) from the
FP32 micro model (gerador_micro_gguf.py), which validates every tensor
bit-exact before writing it.  Kept here, byte for byte:

  * the 28-byte file header and the 21 index entries of 128 bytes
    (nsz_format.rs:115-245);
  * the tile streams of four tensors: output_norm.weight (one partial tile of
    64 weights), blk.0.attn_q.weight (8 full tiles), token_embd.weight (16)
    and blk.0.ffn_down.weight (21 full tiles and one of 256 weights).

Nothing here decodes: the fixture checks the decoder / encoder restatements
(tests/test_nsz.py) by round trip on the reference's bytes.
"""
from __future__ import annotations

import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KEEP = ["output_norm.weight", "blk.0.attn_q.weight", "token_embd.weight", "blk.0.ffn_down.weight"]


def main(src: str) -> None:
    data = np.fromfile(src, np.uint8)
    n = struct.unpack("<I", data[8:12].tobytes())[0]
    out = {"file_header": data[:28].copy(), "entries": data[28:28 + 128 * n].copy()}
    names = []
    for i in range(n):
        e = data[28 + 128 * i:28 + 128 * (i + 1)].tobytes()
        name = e[:64].split(b"\0")[0].decode()
        off, size = struct.unpack("<QQ", e[73:89])
        if name in KEEP:
            key = name.replace(".", "_")
            out[f"stream_{key}"] = data[off:off + size].copy()
            names.append(name)
    assert sorted(names) == sorted(KEEP), names
    np.savez_compressed(os.path.join(HERE, "nsz_golden.npz"), **out)
    print("wrote", {k: v.size for k, v in out.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: {sys.argv[0]} <path of micro_modelo_ignition.nsz>")
    main(sys.argv[1])
