"""Index maps of the chunk-list kernel's shared-memory layout (sdmchat_b200/csrc/rt_scan.cu, rt_lists_kernel), checked
on the host: with k = 16 the write id of (token t, write index i) is held at word t * 16 + (i ^ ((t >> 1) & 15))
(wslot), and the 16-byte staging store puts int4 group e4 at group (e4 & ~3) | ((e4 & 3) ^ (s >> 2)) with its four
elements permuted by s & 3 (perm4), s = (t >> 1) & 15.  Both must give the same word for every element, keep each
token's ids inside its own row, and the 32 tokens of one write index must fall in 32 distinct banks."""


def wslot(e):
    return (e & ~15) | ((e & 15) ^ ((e >> 5) & 15))


def vector_store_word(e):
    """The word the 16-byte staging store writes element e to."""
    e4, u = e >> 2, e & 3
    sq = (e4 >> 3) & 15
    d4 = (e4 & ~3) | ((e4 & 3) ^ (sq >> 2))
    return 4 * d4 + (u ^ (sq & 3))  # perm4: element u moves to position u ^ (sq & 3)


def test_write_id_layout():
    E = 64 * 16
    assert sorted(wslot(e) for e in range(E)) == list(range(E))  # a permutation
    for e in range(E):
        assert wslot(wslot(e)) == e  # its own inverse: the logical index of a word is wslot(word)
        assert wslot(e) >> 4 == e >> 4  # stays in the token's row (entry order by token is unchanged)
        assert vector_store_word(e) == wslot(e)  # the vector and scalar staging paths agree
    for i in range(16):
        for t0 in (0, 32):
            banks = {wslot((t0 + t) * 16 + i) % 32 for t in range(32)}
            assert len(banks) == 32, (i, t0)
