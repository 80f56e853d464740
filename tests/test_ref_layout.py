"""The restated layout of the reference's GPU kernel (oracle/ref_tiles.py) against layouts p2p.compact.Tiles itself
built (tests/golden/tiles_cases.npz): values, masks, offsets and vcap bit-exact. No GPU."""
import numpy as np
import pytest
import torch

from conftest import tiles_blocks
from oracle import ref_tiles


@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_layout_matches_the_reference_tiles(tiles_golden, name):
    lay = ref_tiles.layout(tiles_blocks(tiles_golden, name))
    meta = tiles_golden[name + "_meta"]
    assert [lay["rows"], lay["vcap"], lay["tiles"], lay["chunks"]] == [int(v) for v in meta[2:]]
    assert np.array_equal(lay["vals"].view(torch.int16).numpy().view(np.uint16), tiles_golden[name + "_vals"])
    assert np.array_equal(lay["masks"].numpy(), tiles_golden[name + "_masks"])
    assert np.array_equal(lay["woff"].numpy(), tiles_golden[name + "_woff"])
