"""Configuration 4 proper (bench.py --corpus-mb): the corpus is split into
contiguous document ranges, one per rank, that cover every document once, and
the pooled generation returns the same documents as synth.documents."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_corpus_ranges_partition_the_documents():
    sys.path.insert(0, ROOT)
    import bench

    for n_docs in (1, 16, 100, 16384):
        for world in (1, 2, 3, 4, 8):
            got = [bench.corpus_range(r, world, n_docs) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n_docs
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [hi - lo for lo, hi in got]
            assert max(sizes) - min(sizes) <= 1


def test_pooled_generation_equals_serial():
    sys.path.insert(0, ROOT)
    import bench
    from compress_zip_b200 import synth

    assert bench.corpus_documents(10000, 10260, 2) == synth.documents(range(10000, 10260), 65536)
