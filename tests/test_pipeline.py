"""Host logic of tadma_b200.pipeline (CPU): the row chunks of a step cover
every row exactly once, in order, with no empty chunk."""
from tadma_b200.pipeline import chunk_bounds


def test_chunk_bounds_cover_rows_once():
    for rows in (0, 1, 5, 7, 64, 1000, 8192):
        for chunks in (0, 1, 3, 8, 16, 10000):
            b = chunk_bounds(rows, chunks)
            assert len(b) <= max(1, chunks)
            covered = [r for lo, hi in b for r in range(lo, hi)]
            assert covered == list(range(rows))
            assert all(hi > lo for lo, hi in b)
