"""Seeded synthetic workloads for the fan-out / fan-in path.

The reference publishes no dataset for these ops; its op benchmark
(``scripts/benchmark_mp_ops.py:203-258``) draws seeded random inputs. These
generators produce the shapes and value distributions of the five benchmark
configurations:

* ``cfg1`` - parity micro-workload: N=2000 nodes, D=32, E=20000 messages.
* ``cfg2`` - large op benchmark: N=2**20, E=2**24, D=64, truncated Zipf(1.3)
  destinations, sorted or unsorted.
* ``cfg5`` - skewed stress test: N=2**22, E=2**26, D=32, 64 hub destinations
  with 100k messages each, the rest uniform.
* ``lgan`` - LGAN pool + graph step (sum / mean indexed reductions): 2**17
  entities, 2**20 relation instances of arity 1..3, 4 RR edges per instance,
  D=64 (no reference benchmark exists for these ops; shapes of a planning
  batch).

Everything is drawn from one ``torch.Generator`` per call in a fixed order, so a
seed fully determines a workload on a given device type.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class FanWorkload:
    """Inputs of one fan-out + fan-in pass.

    Fan-out: ``x[x_rows, D]`` gathered by ``src`` into ``out_rows`` slot rows at
    ``flat_dst``. Fan-in: ``msgs[E, D]`` rows ``flat_src`` reduced into
    ``dim_size`` destination rows ``dst``. ``grad_slots`` / ``grad_nodes`` are
    upstream gradients for the backward ops.
    """

    name: str
    x: torch.Tensor
    src: torch.Tensor
    flat_dst: torch.Tensor
    out_rows: int
    msgs: torch.Tensor
    flat_src: torch.Tensor
    dst: torch.Tensor
    dim_size: int
    grad_slots: torch.Tensor
    grad_nodes: torch.Tensor

    @property
    def num_edges(self) -> int:
        return int(self.src.numel())

    @property
    def emb(self) -> int:
        return int(self.x.size(1))

    def to(self, device, dtype: torch.dtype | None = None) -> "FanWorkload":
        def v(t: torch.Tensor) -> torch.Tensor:
            return t.to(device=device, dtype=dtype) if dtype is not None else t.to(device)

        return FanWorkload(
            self.name, v(self.x), self.src.to(device), self.flat_dst.to(device), self.out_rows,
            v(self.msgs), self.flat_src.to(device), self.dst.to(device), self.dim_size,
            v(self.grad_slots), v(self.grad_nodes),
        )


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def cfg1(seed: int = 0, device="cpu", n: int = 2000, emb: int = 32, edges: int = 20000) -> FanWorkload:
    """Parity micro-workload. Draw order: X=randn(N,D); src=randint(N,(E,));
    dst=randint(N,(E,)); msgs=randn(E,D)*sqrt(2); flat_dst=randperm(E);
    grad_slots=randn(E,D); grad_nodes=randn(N,D). flat_src=arange(E)."""

    g = _gen(device, seed)
    kw = dict(device=device, generator=g)
    x = torch.randn(n, emb, dtype=torch.float32, **kw)
    src = torch.randint(0, n, (edges,), dtype=torch.int64, **kw)
    dst = torch.randint(0, n, (edges,), dtype=torch.int64, **kw)
    msgs = torch.randn(edges, emb, dtype=torch.float32, **kw) * math.sqrt(2.0)
    flat_dst = torch.randperm(edges, dtype=torch.int64, **kw)
    grad_slots = torch.randn(edges, emb, dtype=torch.float32, **kw)
    grad_nodes = torch.randn(n, emb, dtype=torch.float32, **kw)
    flat_src = torch.arange(edges, dtype=torch.int64, device=device)
    return FanWorkload("cfg1", x, src, flat_dst, edges, msgs, flat_src, dst, n, grad_slots, grad_nodes)


def zipf_destinations(n: int, edges: int, alpha: float, g: torch.Generator, device) -> torch.Tensor:
    """Truncated Zipf(alpha) node ids: rank k in [1, n] with P(k) ~ k**-alpha,
    sampled with replacement, mapped to node ids through a random permutation."""

    ranks = torch.arange(1, n + 1, dtype=torch.float64, device=device)
    weights = ranks.pow(-float(alpha)).to(torch.float32)
    out = torch.empty(edges, dtype=torch.int64, device=device)
    chunk = 1 << 22  # torch.multinomial caps the sample count per call
    for start in range(0, edges, chunk):
        stop = min(edges, start + chunk)
        out[start:stop] = torch.multinomial(weights, stop - start, replacement=True, generator=g)
    node_of_rank = torch.randperm(n, dtype=torch.int64, device=device, generator=g)
    return node_of_rank[out]


def cfg2(
    seed: int = 0,
    device="cpu",
    sorted_dst: bool = False,
    dtype: torch.dtype = torch.float32,
    n: int = 1 << 20,
    edges: int = 1 << 24,
    emb: int = 64,
    alpha: float = 1.3,
) -> FanWorkload:
    """Large op benchmark: uniform ``src``, Zipf(1.3) ``dst``, values ~N(0,1).

    ``sorted_dst`` stable-sorts the fan-in edges by destination and permutes the
    message rows with them (``flat_src`` stays ``arange``) so segments are
    contiguous; the fan-out slots become ``arange`` (in-order slots). bf16 data
    is generated in float32 and cast.
    """

    g = _gen(device, seed)
    kw = dict(device=device, generator=g)
    x = torch.randn(n, emb, dtype=torch.float32, **kw)
    src = torch.randint(0, n, (edges,), dtype=torch.int64, **kw)
    dst = zipf_destinations(n, edges, alpha, g, device)
    msgs = torch.randn(edges, emb, dtype=torch.float32, **kw)
    flat_dst = torch.randperm(edges, dtype=torch.int64, **kw)
    grad_slots = torch.randn(edges, emb, dtype=torch.float32, **kw)
    grad_nodes = torch.randn(n, emb, dtype=torch.float32, **kw)
    flat_src = torch.arange(edges, dtype=torch.int64, device=device)
    if sorted_dst:
        dst, perm = torch.sort(dst, stable=True)
        msgs = msgs[perm]
        flat_dst = torch.arange(edges, dtype=torch.int64, device=device)
    wl = FanWorkload(
        "cfg2-sorted" if sorted_dst else "cfg2-unsorted",
        x, src, flat_dst, edges, msgs, flat_src, dst, n, grad_slots, grad_nodes,
    )
    return wl.to(device, dtype) if dtype != torch.float32 else wl


def cfg5(
    seed: int = 0,
    device="cpu",
    n: int = 1 << 22,
    edges: int = 1 << 26,
    emb: int = 32,
    hubs: int = 64,
    per_hub: int = 100_000,
) -> FanWorkload:
    """Skewed-degree stress test: 64 hub nodes (seeded ``randperm``) receive
    100 000 messages each, the remaining messages pick uniform destinations;
    the destination order is shuffled. Messages ~N(0, 4)."""

    g = _gen(device, seed)
    kw = dict(device=device, generator=g)
    x = torch.randn(n, emb, dtype=torch.float32, **kw)
    src = torch.randint(0, n, (edges,), dtype=torch.int64, **kw)
    hub_ids = torch.randperm(n, dtype=torch.int64, **kw)[:hubs]
    rest = edges - hubs * per_hub
    dst = torch.cat([hub_ids.repeat_interleave(per_hub), torch.randint(0, n, (rest,), dtype=torch.int64, **kw)])
    dst = dst[torch.randperm(edges, dtype=torch.int64, **kw)]
    msgs = torch.randn(edges, emb, dtype=torch.float32, **kw) * 2.0
    flat_dst = torch.randperm(edges, dtype=torch.int64, **kw)
    grad_slots = torch.randn(edges, emb, dtype=torch.float32, **kw)
    grad_nodes = torch.randn(n, emb, dtype=torch.float32, **kw)
    flat_src = torch.arange(edges, dtype=torch.int64, device=device)
    return FanWorkload("cfg5", x, src, flat_dst, edges, msgs, flat_src, dst, n, grad_slots, grad_nodes)


def algorithmic_bytes(op: str, wl: FanWorkload, elem_bytes: int | None = None) -> int:
    """Compulsory HBM traffic of one op call: each referenced input row read
    once, every int64 index read once, each output row written once. Sort or
    CSR-build traffic is not counted."""

    s = elem_bytes if elem_bytes is not None else wl.x.element_size()
    d = wl.emb
    e = wl.num_edges if op.startswith("fanout") else int(wl.flat_src.numel())
    if op == "fanout_fwd":
        ux = int(torch.unique(wl.src).numel())
        return ux * d * s + 16 * e + wl.out_rows * d * s
    if op == "fanout_bwd":
        return e * d * s + 16 * e + int(wl.x.size(0)) * d * s
    if op in ("fanin_sum_fwd", "fanin_lse_fwd"):
        return e * d * s + 16 * e + wl.dim_size * d * s
    ud = int(torch.unique(wl.dst).numel())
    if op == "fanin_sum_bwd":
        return ud * d * s + 16 * e + e * d * s
    if op == "fanin_lse_bwd":
        return 2 * e * d * s + 2 * ud * d * s + 16 * e
    raise ValueError(op)


# ---- LGAN batches (lgan_pool_reduce / lgan_relation_graph_step) ----------------------


@dataclass
class LganWorkload:
    """Inputs of one LGAN pool + graph step and its backward.

    ``R`` relation instances of arity 1..max_arity own ``S`` slots
    (``slot_to_relation_instance`` = each instance repeated arity times, in
    order); every slot names a uniform random entity of ``N``. TN edges join
    each instance to the entity of its first slot, NN edges to the entities of
    its other slots, RR edges are ``rr_per_relation * R`` uniform instance
    pairs. Upstream gradients ``grad_x [R, D]``, ``grad_tn / grad_nn [N, D]``.
    """

    name: str
    slots: torch.Tensor
    slot_to_rel: torch.Tensor
    arities: torch.Tensor
    rr_src: torch.Tensor
    rr_dst: torch.Tensor
    tn_rel: torch.Tensor
    tn_ent: torch.Tensor
    nn_rel: torch.Tensor
    nn_ent: torch.Tensor
    entity_dim_size: int
    grad_x: torch.Tensor
    grad_tn: torch.Tensor
    grad_nn: torch.Tensor

    @property
    def emb(self) -> int:
        return int(self.slots.size(1))

    @property
    def relation_count(self) -> int:
        return int(self.arities.numel())

    @property
    def num_slots(self) -> int:
        return int(self.slots.size(0))

    def graph(self) -> tuple:
        return (self.rr_src, self.rr_dst, self.tn_rel, self.tn_ent, self.nn_rel, self.nn_ent)

    def to(self, device, dtype: torch.dtype | None = None) -> "LganWorkload":
        def v(t):
            return t.to(device=device, dtype=dtype) if dtype is not None else t.to(device)

        return LganWorkload(
            self.name, v(self.slots), self.slot_to_rel.to(device), self.arities.to(device), self.rr_src.to(device),
            self.rr_dst.to(device), self.tn_rel.to(device), self.tn_ent.to(device), self.nn_rel.to(device),
            self.nn_ent.to(device), self.entity_dim_size, v(self.grad_x), v(self.grad_tn), v(self.grad_nn),
        )


def lgan(seed: int = 0, device="cpu", entities: int = 1 << 17, relations: int = 1 << 20, max_arity: int = 3,
         rr_per_relation: int = 4, emb: int = 64, dtype: torch.dtype = torch.float32) -> LganWorkload:
    """Synthetic LGAN batch (shapes of a planning-domain batch: ~2 slots per
    relation instance, 8x more instances than entities). Draw order: arities,
    slot entities, RR pairs, slot values, the three upstream gradients."""

    g = _gen(device, seed)
    kw = dict(device=device, generator=g)
    R, N = int(relations), int(entities)
    arities = torch.randint(1, int(max_arity) + 1, (R,), dtype=torch.int64, **kw)
    slot_to_rel = torch.repeat_interleave(torch.arange(R, dtype=torch.int64, device=device), arities)
    S = int(slot_to_rel.numel())
    slot_ent = torch.randint(0, N, (S,), dtype=torch.int64, **kw)
    first = torch.ones(S, dtype=torch.bool, device=device)
    first[1:] = slot_to_rel[1:] != slot_to_rel[:-1]
    rr_src = torch.randint(0, R, (int(rr_per_relation) * R,), dtype=torch.int64, **kw)
    rr_dst = torch.randint(0, R, (int(rr_per_relation) * R,), dtype=torch.int64, **kw)
    slots = torch.randn(S, int(emb), dtype=torch.float32, **kw)
    grad_x = torch.randn(R, int(emb), dtype=torch.float32, **kw)
    grad_tn = torch.randn(N, int(emb), dtype=torch.float32, **kw)
    grad_nn = torch.randn(N, int(emb), dtype=torch.float32, **kw)
    wl = LganWorkload(
        "lgan", slots, slot_to_rel, arities, rr_src, rr_dst, slot_to_rel[first], slot_ent[first],
        slot_to_rel[~first], slot_ent[~first], N, grad_x, grad_tn, grad_nn,
    )
    return wl.to(device, dtype) if dtype != torch.float32 else wl


def lgan_algorithmic_bytes(wl: LganWorkload, elem_bytes: int | None = None) -> dict[str, int]:
    """Compulsory HBM traffic of lgan_pool_reduce and its backward (the
    reference's composition: every intermediate row written and read once,
    every distinct gathered row read once, every int64 index read once; the
    pool's slot rows and the arities read once)."""

    s = elem_bytes if elem_bytes is not None else wl.slots.element_size()
    rb = wl.emb * s
    R, N, S = wl.relation_count, wl.entity_dim_size, wl.num_slots
    e_rr, e_tn, e_nn = int(wl.rr_src.numel()), int(wl.tn_rel.numel()), int(wl.nn_rel.numel())

    def uniq(t) -> int:
        return int(torch.unique(t).numel()) if t.numel() else 0

    fwd = (S * rb + 8 * S + 8 * R + R * rb                      # pool: slots, index, arities -> x0
           + uniq(wl.rr_src) * rb + 16 * e_rr + R * rb + R * rb  # x1 = x0 + agg_rr(x0)
           + uniq(wl.tn_rel) * rb + 16 * e_tn + N * rb          # tn = agg(x1)
           + uniq(wl.nn_rel) * rb + 16 * e_nn + N * rb)         # nn = agg(x1)
    bwd = (R * rb + uniq(wl.tn_ent) * rb + 16 * e_tn + R * rb   # g1 = gx + rev_tn(gtn)
           + uniq(wl.nn_ent) * rb + 16 * e_nn + R * rb + R * rb  # g1 += rev_nn(gnn)
           + uniq(wl.rr_dst) * rb + 16 * e_rr + R * rb + R * rb  # g0 = g1 + rev_rr(g1)
           + R * rb + 8 * R + 8 * S + S * rb)                   # grad_slots = g0[s2r] / arity
    return {"lgan_fwd": fwd, "lgan_bwd": bwd}


# ---- relational batches (RelationalGNN workloads) ------------------------------------


@dataclass
class RelationalBatch:
    """A batch of planning states as one disjoint-union relational graph.

    ``relations[p]`` holds the ground atoms of predicate ``p`` as int64
    ``[n_atoms, arity]`` global object ids (arity 0: ``[n_atoms, 0]``); objects
    of state ``s`` are ``object_state == s``. This is the information relmo
    reads from a PyG ``HeteroData`` batch: the edge types
    ``(object, str(pos), predicate)`` / ``(predicate, str(pos), object)`` are
    column ``pos`` of ``relations[predicate]``.
    """

    num_objects: int
    num_states: int
    relations: dict
    object_state: torch.Tensor

    @property
    def arities(self) -> dict:
        return {p: int(a.size(1)) for p, a in self.relations.items()}

    def to(self, device, non_blocking: bool = False) -> "RelationalBatch":
        return RelationalBatch(self.num_objects, self.num_states,
                               {p: a.to(device, non_blocking=non_blocking) for p, a in self.relations.items()},
                               self.object_state.to(device, non_blocking=non_blocking))

    def state_slice(self, lo: int, hi: int) -> "RelationalBatch":
        """States ``[lo, hi)`` as a batch of their own (objects renumbered from 0).
        Objects are stored state-major (``object_state`` non-decreasing) and every
        atom's arguments belong to one state."""

        bounds = torch.searchsorted(self.object_state, torch.tensor([lo, hi], device=self.object_state.device))
        o_lo, o_hi = (int(v) for v in bounds.tolist())
        relations = {}
        for p, args in self.relations.items():
            if args.size(1) == 0:
                relations[p] = args[:0]
                continue
            first = args[:, 0]
            keep = (first >= o_lo) & (first < o_hi)
            relations[p] = args[keep] - o_lo
        return RelationalBatch(o_hi - o_lo, hi - lo, relations, self.object_state[o_lo:o_hi] - lo)


def relational_batch(num_states: int, objects_per_state: int, arities: dict, atoms_per_predicate: int,
                     seed: int = 0, device="cpu") -> RelationalBatch:
    """Synthetic states: every predicate gets ``atoms_per_predicate`` atoms per
    state whose arguments are objects of that state drawn uniformly (seeded)."""

    g = _gen("cpu", seed)
    base = (torch.arange(num_states, dtype=torch.int64) * objects_per_state).view(-1, 1, 1)
    relations = {}
    for pred in sorted(arities):
        k = int(arities[pred])
        args = torch.randint(0, objects_per_state, (num_states, atoms_per_predicate, k), dtype=torch.int64, generator=g)
        relations[pred] = (args + base).reshape(num_states * atoms_per_predicate, k).to(device)
    object_state = torch.arange(num_states, dtype=torch.int64).repeat_interleave(objects_per_state).to(device)
    return RelationalBatch(num_states * objects_per_state, num_states, relations, object_state)


CFG3_ARITIES = {"p0": 0, "p1": 1, "p2": 1, "p3": 2, "p4": 2, "p5": 2, "p6": 3, "p7": 3}
CFG4_ARITIES = {f"p{i:02d}": 1 + (i % 3) for i in range(12)}


def cfg3_batch(seed: int = 0, device="cpu", states: int = 256) -> RelationalBatch:
    """CentralizedRelationalGNN workload: 256 states x 50 objects, 8 predicates of
    arity {0,1,1,2,2,2,3,3}, 50 atoms per predicate (400 ground atoms per state)."""

    return relational_batch(states, 50, CFG3_ARITIES, 50, seed, device)


def cfg4_batch(seed: int = 0, device="cpu", states: int = 4096) -> RelationalBatch:
    """Decentralized RelationalGNN workload: states x 100 objects, 12 predicates of
    arity 1-3 (four each), 125 atoms per predicate (1500 ground atoms per state)."""

    return relational_batch(states, 100, CFG4_ARITIES, 125, seed, device)
