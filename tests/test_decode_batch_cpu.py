"""Batched decode-step driver (cottus_decode_batch_*), host bookkeeping only.

Checked against a host model of Engine::generate's block handling
(engine.cpp:52-95) on the restated reference allocator: a block whenever a
sequence's next position starts one (engine.cpp:73-77), blocks returned in
allocation order (engine.cpp:88-90), LIFO reuse, the first block is 0.
"""
import numpy as np
import pytest

from helpers import BatchReplica

cb = pytest.importorskip("cottus_b200")


def _check_same(batch, rep):
    assert batch.rows() == rep.rows
    assert len(batch) == len(rep.rows)
    assert batch.free_blocks() == rep.alloc.num_free()
    for r, sid in enumerate(rep.rows):
        row, pos, blocks = batch.sequence(sid)
        assert (row, pos, blocks) == (r, rep.seq[sid][0], rep.seq[sid][1])


def test_random_schedule_matches_engine_bookkeeping(oracle):
    rng = np.random.default_rng(5)
    nb, bs, mb, maxb = 40, 16, 7, 12  # 7 rows x 12 blocks > 40: exhaustion happens
    batch = cb.DecodeBatch(nb, bs, mb, maxb)
    rep = BatchReplica(oracle, nb, bs, mb, maxb)
    next_id, ooms = 100, 0
    for step in range(400):
        if len(rep.rows) < mb and rng.random() < 0.3:
            batch.add(next_id)
            rep.add(next_id)
            next_id += 1
        if rep.rows and rng.random() < 0.08:
            sid = int(rng.choice(rep.rows))
            batch.release(sid)
            rep.release(sid)
        # retire sequences that reached the table's length (the reference stops at maxSeqLen)
        for sid in [s for s in rep.rows if rep.seq[s][0] >= maxb * bs]:
            batch.release(sid)
            rep.release(sid)
        ok = rep.begin_step()
        if ok:
            batch.begin_step()
            _check_same(batch, rep)
            batch.end_step()
            rep.end_step()
        else:
            with pytest.raises(cb.CottusError) as e:
                batch.begin_step()
            assert e.value.code == cb.COTTUS_ERR_OUT_OF_MEMORY
            assert "Out of memory" in e.value.message
            ooms += 1
            # nothing changed; free room by ending the oldest sequence
            _check_same(batch, rep)
            sid = rep.rows[0]
            batch.release(sid)
            rep.release(sid)
        _check_same(batch, rep)
    assert next_id > 130 and ooms > 0  # the schedule exercised churn and exhaustion


def test_single_sequence_like_generate(oracle):
    """One sequence through prompt + generation: blocks 0, 1, 2, ... on a fresh
    pool; all returned at the end; a second sequence reuses them LIFO."""
    batch = cb.DecodeBatch(16, 16, 2, 16)
    batch.add(1)
    for _ in range(40):
        batch.begin_step()
        batch.end_step()
    assert batch.sequence(1) == (0, 40, [0, 1, 2])
    batch.release(1)
    assert batch.free_blocks() == 16
    batch.add(2)
    batch.begin_step()
    # freed in allocation order 0, 1, 2 -> the LIFO top is 2
    assert batch.sequence(2) == (0, 0, [2])
    batch.end_step()


def test_exhaustion_undoes_the_step():
    batch = cb.DecodeBatch(3, 16, 4, 8)
    for s in range(4):
        batch.add(s)
    with pytest.raises(cb.CottusError) as e:
        batch.begin_step()  # four rows need a block each, three exist
    assert e.value.code == cb.COTTUS_ERR_OUT_OF_MEMORY
    assert batch.free_blocks() == 3
    assert all(batch.sequence(s)[2] == [] for s in range(4))
    batch.release(3)
    batch.begin_step()
    assert batch.free_blocks() == 0
    assert [batch.sequence(s)[2] for s in range(3)] == [[0], [1], [2]]
    batch.end_step()


def test_length_limit_and_errors():
    batch = cb.DecodeBatch(8, 16, 2, 2)
    batch.add(7)
    for _ in range(32):
        batch.begin_step()
        batch.end_step()
    with pytest.raises(cb.CottusError) as e:
        batch.begin_step()  # position 32 needs a third block; the table has two columns
    assert e.value.code == cb.COTTUS_ERR_OUT_OF_RANGE
    with pytest.raises(cb.CottusError) as e:
        batch.add(7)
    assert e.value.code == cb.COTTUS_ERR_INVALID_ARGUMENT
    with pytest.raises(cb.CottusError) as e:
        batch.release(8)
    assert e.value.code == cb.COTTUS_ERR_INVALID_ARGUMENT
    batch.add(8)
    with pytest.raises(cb.CottusError) as e:
        batch.add(9)
    assert e.value.code == cb.COTTUS_ERR_OUT_OF_RANGE  # batch full
    batch.release(7)
    batch.begin_step()
    with pytest.raises(cb.CottusError):
        batch.add(10)  # inside a step
    with pytest.raises(cb.CottusError):
        batch.release(8)
    with pytest.raises(cb.CottusError):
        batch.begin_step()
    batch.end_step()
    with pytest.raises(cb.CottusError):
        batch.end_step()


def test_bad_descriptors():
    for args in [(0, 16, 2, 2), (8, 0, 2, 2), (8, 16, 0, 2), (8, 16, 2, 0), (8, 16, 1 << 16, 1 << 16)]:
        with pytest.raises(cb.CottusError) as e:
            cb.DecodeBatch(*args)
        assert e.value.code == cb.COTTUS_ERR_INVALID_ARGUMENT
