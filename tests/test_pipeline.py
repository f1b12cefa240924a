"""Host logic of tadma_b200.pipeline (CPU): the row chunks of a step cover
every row exactly once, in order, with no empty chunk; the ramped layout
shrinks the first and the last chunk."""
from tadma_b200.pipeline import chunk_bounds, ramped_bounds


def _covers(b, rows):
    covered = [r for lo, hi in b for r in range(lo, hi)]
    return covered == list(range(rows)) and all(hi > lo for lo, hi in b)


def test_chunk_bounds_cover_rows_once():
    for rows in (0, 1, 5, 7, 64, 1000, 8192):
        for chunks in (0, 1, 3, 8, 16, 10000):
            b = chunk_bounds(rows, chunks)
            assert len(b) <= max(1, chunks)
            assert _covers(b, rows)


def test_ramped_bounds_cover_rows_once_with_small_ends():
    for rows in (1, 2, 5, 7, 64, 1000, 8192):
        for chunks in (1, 2, 3, 8, 16):
            for part in (2, 4, 8):
                b = ramped_bounds(rows, chunks, part)
                assert _covers(b, rows), (rows, chunks, part, b)
                assert len(b) <= max(1, chunks) + 2
    b = ramped_bounds(8192, 8, 4)
    assert [hi - lo for lo, hi in b] == [256, 768] + [1024] * 6 + [768, 256]
