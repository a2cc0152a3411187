"""The benchmark's workload generators and mask-aware pair counts (CPU).

``bench.py`` reports mask-aware TFLOP/s: FLOPs are the reference formula
(``reference.py:338-356``) over the exact count of allowed (query, key) pairs,
vision-future and document restrictions included.  Its closed-form counter is
checked here against the oracle's dense count of the same mask, and the
generators against the shapes BASELINE.json describes."""

import numpy as np
import pytest

import bench
import oracle


@pytest.mark.parametrize("seed", range(6))
def test_local_pair_count_matches_the_dense_mask(seed):
    rng = np.random.default_rng(seed)
    s, w = int(rng.integers(50, 400)), int(rng.integers(1, 80))
    vis = np.full(s, -1, np.int64)
    for i in range(int(rng.integers(0, 5))):
        a = int(rng.integers(0, s - 10))
        vis[a:a + int(rng.integers(1, 40))] = i % 3  # ids may repeat, spans may touch
    cuts = np.sort(rng.choice(np.arange(1, s), size=int(rng.integers(0, 3)), replace=False))
    doc = np.zeros(s, np.int64)
    for j, c in enumerate(cuts):
        doc[c:] = j + 1
    want = oracle.mask_aware_pairs(q_len=s, kv_len=s, sliding_window=w, vision_block_ids=vis,
                                   document_ids=doc, allow_vision_bidirectional=True)
    assert bench.local_pairs(vis, doc, w) == want


def test_text_pairs_match_the_reference_counts():
    assert bench.text_pairs(2048, 1024) == 1_573_376   # configs[0]
    assert bench.text_pairs(4096, 0) == 8_390_656      # configs[1]
    assert bench.text_pairs(262144, 0) == 34_359_869_440  # configs[4](i)


def test_c2_generator_places_six_images_per_sequence():
    vis = bench.c2_metadata()
    assert vis.shape == (2, 8192)
    for b in range(2):
        ids, counts = np.unique(vis[b][vis[b] >= 0], return_counts=True)
        assert ids.tolist() == list(range(6)) and counts.tolist() == [256] * 6
        # each image is one contiguous run, so its future pairs are 256*255/2
        assert bench.local_pairs(vis[b], None, 1024) == 7_864_832 + 6 * 32_640


def test_c3_packing_shape_and_vision_share():
    lens, cu, doc, vis = bench.c3_packing()
    assert cu[-1] == 131072 and cu[0] == 0 and len(lens) == len(cu) - 1
    assert all(1 <= n <= 32768 for n in lens)
    assert 0.045 <= (vis >= 0).mean() <= 0.055
    for a, b in zip(cu[:-1], cu[1:]):  # images stay inside their segment (document)
        seg = vis[a:b]
        assert (seg >= 0).sum() % 256 == 0


def test_peak_choice_follows_the_window_clocks():
    """A line's fraction is taken against the burst peak only for a short window
    at full clock with no power capping; otherwise against the sustained one."""
    peaks = (1400.0, 1660.0, "measured")
    full = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    capped = {"sm_mhz": 1250.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    slow = {"sm_mhz": 1500.0, "sm_max_mhz": 1965.0, "reasons": []}
    assert bench.pick_peak(peaks, full, 0.5)[0] == 1660.0
    assert "burst" in bench.pick_peak(peaks, full, 0.5)[1]
    assert bench.pick_peak(peaks, full, 30.0)[0] == 1400.0  # long window
    assert bench.pick_peak(peaks, capped, 0.5)[0] == 1400.0
    assert bench.pick_peak(peaks, slow, 0.5)[0] == 1400.0
    assert bench.pick_peak(peaks, {"sm_mhz": None, "sm_max_mhz": None, "reasons": []},
                           0.5)[0] == 1400.0  # no samples: the conservative figure
