"""Index bookkeeping of the weight-streaming kernel's cluster reduction (csrc/matmul_tc.cu, matmul_stream_kernel),
restated on the CPU: group j = (m tile, n tile, lane) of a CTA's fp32 sums goes to CTA owner(j) of the cluster, into
slot slot_of(j) of the sender's region there. Every owner must receive each of its groups in a distinct slot below
per_owner, and the qkv epilogue's ownership must keep a row's columns (rows g and g + 8 of an m tile) in one CTA."""
import itertools

import pytest


def owner(j, S, epi):
    return ((j & 31) >> 2) % S if epi else j % S


def slot_of(j, S, epi):
    return (j >> 5) * (32 // S) + (((j & 31) >> 2) // S) * 4 + (j & 3) if epi else j // S


def row_col(j, NT):
    lane, t = j & 31, j >> 5
    mt, nt = t // NT, t % NT
    return mt * 16 + (lane >> 2), nt * 8 + 2 * (lane & 3)


@pytest.mark.parametrize("MT,NT,S,epi", [(mt, nt, s, e) for mt, nt, s, e in itertools.product(
    (1, 2, 4), (1, 2, 3, 4, 5, 6, 7, 8, 16), (1, 2, 4, 8), (0, 1)) if mt * nt <= 32 and (not e or nt == 16)])
def test_every_group_has_one_slot_at_its_owner(MT, NT, S, epi):
    G = MT * NT * 32
    per_owner = (G + S - 1) // S
    seen = {}
    for j in range(G):
        key = (owner(j, S, epi), slot_of(j, S, epi))
        assert 0 <= key[0] < S and 0 <= key[1] < per_owner, (j, key)
        assert key not in seen, (j, seen.get(key), key)
        seen[key] = j
    if epi:
        # all columns of a row belong to one CTA, and that CTA is rank row mod S (the epilogue's row loop)
        for j in range(G):
            row, _ = row_col(j, NT)
            assert owner(j, S, epi) == row % S
        # the up partner of a gate group (swiglu form: + 16 NT) has the same owner in the plain form
    for j in range(G):
        partner = j + 16 * NT
        if not epi and NT % 2 == 0 and partner < G and (j >> 5) % NT < NT // 2:
            assert owner(partner, S, 0) == owner(j, S, 0)
