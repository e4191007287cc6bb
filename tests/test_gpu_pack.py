"""Pack ops on the GPU (their index arithmetic and concatenation as one device
pass per 64 parts): torch.ops.relm_mp.*pack* and the C ABI
relm_mp_pack_index against the reference library's own outputs
(tests/golden/ref_pack.npz, made from mp_ops.cpp:412-570, 2511-2773 by
tests/golden/make_golden.py) and against its ATen formulas (relmo
src/relmo/ops/mp_pack.py:66-292, restated in relmo_b200/ops/mp_pack.py) —
bit-exact, with empty parts, strided parts and more than one launch's worth
(64) of parts; argument errors with the reference's messages."""

from __future__ import annotations

import pytest
import torch

import re

import numpy as np

from relmo_b200 import capi
from relmo_b200.ops import mp, mp_pack
from tests._golden import load_pack_cases

PACK_CASES = load_pack_cases()

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _load_library():
    assert mp.available(), "relm_mp library not loadable"


def _parts(n_parts, seed, device="cuda", max_len=300):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(0, max_len, (n_parts,), generator=g).tolist()
    lens[0] = max(lens[0], 1)
    if n_parts > 2:
        lens[1] = 0  # an empty part
    return [torch.randint(0, 1000, (2 * n,), generator=g)[::2].to(device) for n in lens]  # strided


@pytest.mark.parametrize("n_parts", [1, 3, 64, 65, 150])
def test_pack_index_capi(n_parts):
    parts = _parts(n_parts, n_parts)
    muls = [1 + (i % 3) for i in range(n_parts)]
    adds = [7 * i for i in range(n_parts)]
    got = capi.pack_index(parts, muls, adds)
    expect = torch.cat([p * m + a for p, m, a in zip(parts, muls, adds)])
    assert torch.equal(got, expect)


@pytest.mark.parametrize("n_parts", [1, 5, 70])
def test_pack_multi_ops_match_formulas(n_parts):
    g = torch.Generator().manual_seed(3)
    idx = _parts(n_parts, 10 + n_parts)
    idx2 = _parts(n_parts, 20 + n_parts)
    idx2 = [b[: a.numel()] if b.numel() >= a.numel() else torch.cat([b, b.new_zeros(a.numel() - b.numel())])
            for a, b in zip(idx, idx2)]
    vals = [torch.randn(int(torch.randint(1, 50, (1,), generator=g)), 4, device="cuda") for _ in range(n_parts)]
    for op, ref in [("fanout_pack_multi", mp_pack.fanout_pack_multi_python),
                    ("fanin_pack_multi", mp_pack.fanin_pack_multi_python)]:
        got = getattr(torch.ops.relm_mp, op)(vals, idx, idx2)
        expect = ref(vals, idx, idx2)
        for a, b in zip(got, expect):
            assert torch.equal(a, b), op


@pytest.mark.parametrize("mode", [0, 1])
def test_pack_from_edges_ops_match_formulas(mode):
    g = torch.Generator().manual_seed(5 + mode)
    n_vals, n_edges = 4, 40
    vals = [torch.randn(int(torch.randint(1, 60, (1,), generator=g)), 8, device="cuda") for _ in range(n_vals)]
    es = _parts(n_edges, 30 + mode)
    ed = [torch.randint(0, 90, (e.numel(),), generator=g).cuda() for e in es]
    part_ids = torch.randint(0, n_vals, (n_edges,), generator=g).tolist()
    arity = [1 + (i % 3) for i in range(n_edges)]
    pos = [i % a for i, a in enumerate(arity)]
    slots = [11 * i for i in range(n_edges)]
    got = torch.ops.relm_mp.fanout_pack_from_edges(vals, es, ed, part_ids, arity, pos, slots)
    expect = mp_pack.fanout_pack_from_edges_python(vals, es, ed, part_ids, arity, pos, slots)
    for a, b in zip(got, expect):
        assert torch.equal(a, b)
    got = torch.ops.relm_mp.fanin_pack_from_edges(vals, es, ed, part_ids, arity, pos, mode)
    expect = mp_pack.fanin_pack_from_edges_python(vals, es, ed, part_ids, arity, pos, mode)
    for a, b in zip(got, expect):
        assert torch.equal(a, b)


@pytest.mark.parametrize("case", PACK_CASES, ids=[c.name for c in PACK_CASES])
def test_pack_ops_equal_reference_library_on_cuda(case):
    args = []
    for a in case.args:
        if isinstance(a, list) and a and isinstance(a[0], np.ndarray):
            args.append([torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in a])
        else:
            args.append(a)
    op = getattr(torch.ops.relm_mp, case.op)
    if case.raises:
        with pytest.raises(Exception, match=re.escape(case.message)):
            op(*args)
        return
    got = op(*args)
    for g, ref in zip(got, case.outs):
        assert g.is_cuda and g.dtype == torch.from_numpy(ref).dtype
        assert np.array_equal(g.cpu().numpy(), ref), case.name
