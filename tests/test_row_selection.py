"""The row selector of the large-size GPU parity tests (tests/gpu_util.coverage_rows). CPU only."""

from __future__ import annotations

import numpy as np

from oracle import moe_oracle as orc
from tests.gpu_util import coverage_rows


def test_coverage_rows_cover_every_tile_index(pkg):
    from muse_moe_w4a16_b200 import synth
    shape = synth.CONFIGS["cfg5"]
    data = synth.baseline_input(shape, 4096, seed=1)
    ids = data["topk_ids"].numpy()
    rows = coverage_rows(ids, 0, 256, 128, 64, seed=1)
    offsets, order, row_of = orc.route(ids, 0, 256)
    counts = np.diff(offsets)
    hot = int(np.argmax(counts))
    tiles_hit = set()
    for t in rows:
        for s in range(ids.shape[1]):
            r = row_of[t * ids.shape[1] + s]
            if offsets[hot] <= r < offsets[hot + 1]:
                tiles_hit.add((r - offsets[hot]) // 128)
    assert tiles_hit == set(range(-(-int(counts[hot]) // 128)))
