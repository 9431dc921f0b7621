"""The oracle's restatement of the reference's speculative acceptance loop
(engine/generate.py:130-169) on hand-worked cases that follow the reference's steps."""


def test_first_mismatch_rewinds_rejected_suffix(oracle):
    # candidates [t, d0, d1, d2, d3]; verified [v0..v4]; comparable [t, v0, v1, v2, v3]
    emitted, nxt, rw, drw, fin = oracle.spec_accept_ref([7, 1, 2, 3, 4], [1, 2, 9, 5, 6])
    # i=0: t == t, i=1: v0=1 == d0, i=2: v1=2 == d1, i=3: v2=9 != d2=3 -> rejected 5-3 = 2
    assert emitted == [7, 1, 2] and nxt == 9 and (rw, drw) == (2, 1) and not fin




def test_all_accepted(oracle):
    emitted, nxt, rw, drw, fin = oracle.spec_accept_ref([7, 1, 2, 3], [1, 2, 3, 8])
    assert emitted == [7, 1, 2, 3] and nxt == 8 and (rw, drw) == (0, 0) and not fin


def test_first_draft_rejected(oracle):
    emitted, nxt, rw, drw, fin = oracle.spec_accept_ref([7, 1, 2, 3], [5, 2, 3, 8])
    assert emitted == [7] and nxt == 5 and (rw, drw) == (3, 2) and not fin


def test_end_of_sequence_and_budget(oracle):
    # an emitted eos finishes the request without being emitted
    assert oracle.spec_accept_ref([7, 0, 2], [0, 2, 4], eos_id=0)[0] == [7]
    assert oracle.spec_accept_ref([7, 0, 2], [0, 2, 4], eos_id=0)[4]
    # a rejected position whose verified token is eos finishes after the rewind
    emitted, nxt, rw, drw, fin = oracle.spec_accept_ref([7, 1, 2], [0, 2, 4], eos_id=0)
    assert emitted == [7] and nxt == 0 and rw == 2 and fin
    # budget: stop right after the budget-th emitted token
    emitted, nxt, rw, drw, fin = oracle.spec_accept_ref([7, 1, 2, 3], [1, 2, 3, 8], budget=2)
    assert emitted == [7, 1] and nxt is None and fin
