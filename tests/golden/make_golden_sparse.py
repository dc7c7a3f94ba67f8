"""Golden fixtures for the mask-aware sparse pattern, from the reference's own code.

    python tests/golden/make_golden_sparse.py /path/to/reference

Imports ``layers/attention/backends/mask_sta.py`` from the reference (with the
diffusers stub of ``make_golden.py``) and runs its ``block_geometry``,
``protected_blocks`` and ``block_table`` on the CPU, for an empty mask, a
one-cell mask and the seeded synthetic ellipse mask of the sparse benchmark
configuration.  Writes ``mask_sta_golden.npz`` (compressed; bool arrays
bit-packed).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from make_golden import install_diffusers_stub  # noqa: E402

from eraserdit_b200.sparse_pattern import ellipse_masks  # noqa: E402


def main(reference: Path) -> None:
    install_diffusers_stub()
    sys.path.insert(0, str(reference))
    from layers.attention.backends import mask_sta as ref

    permutation, background = ref.block_geometry("cpu")
    out = dict(permutation=permutation.numpy().astype(np.int32),
               background=np.packbits(background.numpy()), background_shape=background.shape)
    ellipse = ellipse_masks(ref.GRID, seed=3)
    one = torch.zeros(ref.GRID)
    one[0, 10, 10] = 0.0039
    for name, m in (("ellipse", ellipse.float()), ("one_cell", one),
                    ("empty", torch.zeros(ref.GRID))):
        query, binary, expanded = ref.protected_blocks(m.view(1, 1, *ref.GRID), permutation)
        table = background.clone()
        table[query] = True
        lut, counts = ref.block_table(table)
        out[f"{name}_mask"] = np.packbits(binary.flatten().numpy())
        out[f"{name}_expanded"] = np.packbits(expanded.flatten().numpy())
        out[f"{name}_protected"] = query.numpy()
        out[f"{name}_lut"] = lut.numpy().astype(np.int16)
        out[f"{name}_counts"] = counts.numpy().astype(np.int32)
    np.savez_compressed(HERE / "mask_sta_golden.npz", **out)
    print("wrote", HERE / "mask_sta_golden.npz")


if __name__ == "__main__":
    main(Path(sys.argv[1]))
