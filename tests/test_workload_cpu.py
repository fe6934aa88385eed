"""CPU tests of the benchmark workload definitions: the five configurations'
shapes and algorithmic bytes, and the rows the full-size parity checks sample
(tests/test_configs_full.py and bench.py's `parity` field)."""
import pytest

import kvdecode as kvd
import workload as wl


def test_configurations_match_the_north_star_shapes():
    c = wl.CONFIGS
    assert (c[1].batch, c[1].q_heads, c[1].kv_heads, c[1].head_dim, c[1].seq_len) == (1, 8, 8, 64, 1024)
    assert (c[2].batch, c[2].q_heads, c[2].kv_heads, c[2].head_dim, c[2].seq_len) == (64, 32, 32, 128, 4096)
    assert (c[3].batch, c[3].q_heads, c[3].kv_heads, c[3].head_dim, c[3].seq_len) == (4, 32, 32, 128, 131072)
    assert (c[4].batch, c[4].q_heads, c[4].head_dim, c[4].ragged, c[4].append) == (128, 32, 128, (256, 8192), True)
    assert (c[5].batch, c[5].q_heads, c[5].kv_heads, c[5].head_dim, c[5].seq_len) == (256, 64, 8, 128, 2048)
    assert wl.step_bytes(c[2]) == 2_216_689_664
    assert wl.step_bytes(c[5]) == 1_124_073_472


def test_ragged_lengths_are_seeded_and_in_range():
    a = wl.ragged_lengths(wl.CONFIGS[4], 17)
    assert a == wl.ragged_lengths(wl.CONFIGS[4], 17) and len(a) == 128
    assert min(a) >= 256 and max(a) <= 8192
    # configuration 4's bytes: every (sequence, kv head) after its one appended token, plus the append
    lens = [n + 1 for n in a]
    assert wl.step_bytes(wl.CONFIGS[4], lens) == (kvd.algorithmic_bytes(128, 32, 32, 128, lens)
                                                  + 128 * 32 * (2 * 128 * 4 + 2 * (128 + 4)))


@pytest.mark.parametrize("cid", [2, 3, 5])
def test_dense_parity_sample_covers_the_edges(cid):
    cfg = wl.CONFIGS[cid]
    items = wl.parity_items(cfg, cfg.batch)
    assert len(items) == len(set(items))
    assert len(items) * cfg.group >= 64  # at least 64 query rows
    assert (0, 0) in items and (cfg.batch - 1, cfg.kv_heads - 1) in items
    assert all(0 <= b < cfg.batch and 0 <= h < cfg.kv_heads for b, h in items)
    assert items == wl.parity_items(cfg, cfg.batch)  # seeded


def test_ragged_parity_sample_holds_the_longest_and_shortest_sequence():
    cfg = wl.CONFIGS[4]
    lens = wl.ragged_lengths(cfg, 17)
    items = wl.parity_items(cfg, cfg.batch, lens)
    seqs = {b for b, _ in items}
    assert lens.index(max(lens)) in seqs and lens.index(min(lens)) in seqs
    assert 0 in seqs and cfg.batch - 1 in seqs and len(items) >= 64


def test_small_configuration_sample_takes_every_row():
    cfg = wl.CONFIGS[1]
    items = wl.parity_items(cfg, cfg.batch)
    assert sorted(items) == [(0, h) for h in range(cfg.kv_heads)]
