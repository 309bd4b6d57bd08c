"""Host-side pieces of bench.py that need no GPU: the z / lm_head pass split
(it must mirror the library's run_z_phase: passes of at most 256 X rows, as
equal as the 16-row MMA granularity allows) and the roofline byte counts."""
import bench


def test_zlm_passes_split_rows_evenly():
    cases = {16: (16, 1), 80: (80, 1), 120: (128, 1), 256: (256, 1), 257: (144, 2), 272: (144, 2),
             320: (160, 2), 480: (240, 2), 512: (256, 2), 513: (176, 3)}
    for rows, expect in cases.items():
        n, passes = bench.zlm_passes(rows)
        assert (n, passes) == expect, rows
        assert n % 16 == 0 and n <= 256 and n * passes >= rows
        assert n * (passes - 1) < rows  # no empty pass


def test_fc2_and_step_bytes_at_the_headline_shape():
    # fc2: V·E·2 + B·V·2 per launch (3.734 GB at H = G = 4096, E = 12288, B = 1)
    assert bench.fc2_bytes(1, 12288, 151936) == 151936 * 12288 * 2 + 151936 * 2
    # one block moves 60.28 GB at that shape
    b = bench.algorithmic_bytes(1, 4096, 4096, 12288, 151936, 15, 0)
    assert abs(b / 1e9 - 60.28) < 0.01
