"""Topology planner: which ranks form a recoverable replica, and where each
rank's state can be recovered from.

Inputs are the actual process groups of a job: dense data-parallel groups,
expert data-parallel groups, and the non-DP execution groups (TP, PP, CP, EP,
ETP, ...).  Ranks joined (transitively) by execution groups must fail and be
replaced together, so the connected components of the execution groups are
the candidate replicas.  A candidate set is usable for SHIFT-style recovery
when there are at least two replicas of equal size, each covering the same
set of local roles exactly once, no execution group crosses replicas, and
every rank has exactly one same-role source in every other replica that sits
in both its dense-DP and its expert-DP group (so dense and expert state can be
copied from one peer).  With a rank -> node map the planner also reports
which replicas survive each node failure.

Same questions and result fields as shift_full/topology.py:102-402; the
power-of-two rank orders are fixed by Megatron's conventions (dense
``tp + TP*(dp + DP*pp)``, expert ``etp + ETP*(ep + EP*(edp + EDP*pp))``),
and ``node_local_pp`` swaps rank bits 2 and 3 so each 8-rank node holds a
whole replica.  ``box_layout`` adds the layouts this framework runs on one
8-GPU box.
"""
from __future__ import annotations

from collections.abc import Mapping, Sequence

TABLE_4_2 = {
    "A": {"tp": 2, "pp": 2, "ep": 4, "etp": 1},
    "B": {"tp": 4, "pp": 2, "ep": 2, "etp": 1},
    "C": {"tp": 2, "pp": 1, "ep": 4, "etp": 1},
    "D": {"tp": 2, "pp": 1, "ep": 2, "etp": 1},
}

DP_NAMES = {"DP", "DENSE_DP", "EXPERT_DP", "EDP"}


class TopologyError(ValueError):
    """Malformed topology input or an unsupported generated layout."""


def _pow2(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v > 0 and (v & (v - 1)) == 0


def _partition(label: str, groups, world: int) -> tuple:
    """Validate that ``groups`` partitions range(world); return sorted tuples."""
    if groups is None:
        raise TopologyError(f"{label} groups are required")
    try:
        glist = [list(g) for g in groups]
    except TypeError as e:
        raise TopologyError(f"{label} groups must be an iterable of rank groups") from e
    if not glist:
        raise TopologyError(f"{label} groups are empty")
    seen: dict[int, int] = {}
    out = []
    for gi, g in enumerate(glist):
        if not g:
            raise TopologyError(f"{label} group {gi} is empty")
        local = set()
        for r in g:
            if not isinstance(r, int) or isinstance(r, bool) or not 0 <= r < world:
                raise TopologyError(f"{label} group {gi} has out-of-range rank {r!r}")
            if r in local:
                raise TopologyError(f"{label} group {gi} repeats rank {r}")
            if r in seen:
                raise TopologyError(f"{label} groups overlap at rank {r} (groups {seen[r]} and {gi})")
            seen[r] = gi
            local.add(r)
        out.append(tuple(sorted(local)))
    missing = sorted(set(range(world)) - set(seen))
    if missing:
        raise TopologyError(f"{label} groups omit ranks {missing}")
    return tuple(sorted(out))


class _UnionFind:
    def __init__(self, n):
        self.p = list(range(n))

    def find(self, a):
        while self.p[a] != a:
            self.p[a] = self.p[self.p[a]]
            a = self.p[a]
        return a

    def union(self, a, b):
        ra, rb = self.find(a), self.find(b)
        if ra != rb:
            self.p[max(ra, rb)] = min(ra, rb)


def analyze_topology(world_size, dense_dp_groups, expert_dp_groups, execution_groups, rank_to_node=None) -> dict:
    if not isinstance(world_size, int) or isinstance(world_size, bool) or world_size < 1:
        raise TopologyError("world_size must be a positive integer")
    W = world_size
    dense = _partition("dense_dp", dense_dp_groups, W)
    expert = _partition("expert_dp", expert_dp_groups, W)
    if not isinstance(execution_groups, Mapping) or not execution_groups:
        raise TopologyError("execution_groups must be a non-empty name-to-groups mapping")
    execution: dict[str, tuple] = {}
    for raw, groups in execution_groups.items():
        name = str(raw).upper()
        if name in DP_NAMES:
            raise TopologyError(f"{name} is a DP family, not a non-DP execution dependency")
        if name in execution:
            raise TopologyError(f"duplicate execution group name {name}")
        execution[name] = _partition(f"execution {name}", groups, W)

    uf = _UnionFind(W)
    for groups in execution.values():
        for g in groups:
            for r in g[1:]:
                uf.union(g[0], r)
    comp: dict[int, list] = {}
    for r in range(W):
        comp.setdefault(uf.find(r), []).append(r)
    replicas_ranks = sorted((tuple(sorted(v)) for v in comp.values()), key=lambda t: t[0])
    rep_of = {r: i for i, rs in enumerate(replicas_ranks) for r in rs}
    names = sorted(execution)
    pos = {r: {} for r in range(W)}
    for n in names:
        for g in execution[n]:
            for i, r in enumerate(g):
                pos[r][n] = i
    role = {r: tuple(pos[r][n] for n in names) for r in range(W)}

    checks: dict = {}
    rejections: list = []
    n_rep = len(replicas_ranks)
    checks["at_least_two_replicas"] = {"pass": n_rep >= 2, "actual": n_rep}
    if n_rep < 2:
        rejections.append("fewer than two candidate replicas; fail-stop recovery is unavailable")
    sizes = [len(rs) for rs in replicas_ranks]
    checks["equal_replica_sizes"] = {"pass": len(set(sizes)) == 1, "sizes": sizes}
    if len(set(sizes)) != 1:
        rejections.append(f"candidate replica sizes differ: {sizes}")
    role_sets, dup = [], []
    for i, rs in enumerate(replicas_ranks):
        roles = [role[r] for r in rs]
        if len(set(roles)) != len(roles):
            dup.append(i)
        role_sets.append(set(roles))
    same = bool(role_sets) and all(s == role_sets[0] for s in role_sets[1:]) and not dup
    checks["role_coverage_matches"] = {"pass": same, "role_counts": [len(s) for s in role_sets],
                                       "duplicate_role_replicas": dup}
    if not same:
        rejections.append("replicas do not have unique, identical local-role coverage")
    cut = []
    for n, groups in execution.items():
        for g in groups:
            touched = sorted({rep_of[r] for r in g})
            if len(touched) != 1:
                cut.append({"group": n, "ranks": list(g), "replicas": touched})
    checks["execution_groups_unbroken"] = {"pass": not cut, "groups": cut}
    if cut:
        rejections.append("an execution group crosses candidate replica boundaries")

    dense_of = {r: g for g in dense for r in g}
    expert_of = {r: g for g in expert for r in g}
    inter = {r: sorted(set(dense_of[r]) & set(expert_of[r])) for r in range(W)}
    sources, issues = {}, []
    for r in range(W):
        per = {}
        for other in range(n_rep):
            if other == rep_of[r]:
                continue
            cands = [s for s in inter[r] if rep_of[s] == other and role[s] == role[r]]
            per[other] = cands[0] if len(cands) == 1 else cands
            if len(cands) != 1:
                issues.append({"rank": r, "target_replica": other, "candidates": cands})
        sources[r] = per
    checks["recovery_sources_complete"] = {"pass": not issues and n_rep >= 2, "issues": issues}
    if issues:
        rejections.append("missing or ambiguous dense∩expert same-role source in another replica")

    survivable, crossing = {}, {}
    if rank_to_node is not None:
        if isinstance(rank_to_node, Mapping):
            nodes = dict(rank_to_node)
        elif isinstance(rank_to_node, Sequence) and not isinstance(rank_to_node, (str, bytes)):
            if len(rank_to_node) != W:
                raise TopologyError("rank_to_node sequence must have one entry per rank")
            nodes = dict(enumerate(rank_to_node))
        else:
            raise TopologyError("rank_to_node must be a rank mapping or a node sequence")
        missing = sorted(set(range(W)) - set(nodes))
        invalid = sorted(r for r in nodes if r not in range(W))
        if missing or invalid:
            raise TopologyError(f"rank_to_node mismatch: missing={missing}, invalid={invalid}")
        for node in sorted(set(nodes.values()), key=str):
            survivable[node] = [i for i, rs in enumerate(replicas_ranks) if all(nodes[r] != node for r in rs)]
        crossing = {n: sum(len({nodes[r] for r in g}) > 1 for g in groups) for n, groups in execution.items()}

    def gsizes(groups):
        return sorted(len(g) for g in groups)

    return {
        "valid": all(c["pass"] for c in checks.values()),
        "world_size": W,
        "candidate_replica_count": n_rep,
        "replicas": [{"id": i, "ranks": list(rs), "size": len(rs), "role_count": len(role_sets[i])}
                     for i, rs in enumerate(replicas_ranks)],
        "rank_to_replica": rep_of,
        "rank_to_localrole": {r: dict(pos[r]) for r in range(W)},
        "recovery_sources": sources,
        "dense_expert_intersections": inter,
        "survivable_replicas_by_node_failure": survivable,
        "execution_groups_crossing_nodes": crossing,
        "checks": checks,
        "rejections": rejections,
        "metrics": {"dense_dp_group_sizes": gsizes(dense), "expert_dp_group_sizes": gsizes(expert),
                    "dense_expert_intersection_sizes": {r: len(m) for r, m in inter.items()},
                    "execution_group_sizes": {n: gsizes(g) for n, g in execution.items()}},
        "groups": {"dense_dp": [list(g) for g in dense], "expert_dp": [list(g) for g in expert],
                   "execution": {n: [list(g) for g in gs] for n, gs in execution.items()}},
    }


def _vary(coords: dict, axis: str) -> list:
    """Groups of ranks that differ only along ``axis``."""
    buckets: dict = {}
    for r, c in coords.items():
        key = tuple(sorted((k, v) for k, v in c.items() if k != axis))
        buckets.setdefault(key, []).append(r)
    return [sorted(g) for g in buckets.values()]


def make_power2_layout(world_size, tp, pp, ep, etp, cp=1, rank_to_node=None) -> dict:
    for name, v in (("world_size", world_size), ("tp", tp), ("pp", pp), ("ep", ep), ("etp", etp), ("cp", cp)):
        if not _pow2(v):
            raise TopologyError(f"{name}={v!r} must be a positive power of two")
    if cp != 1:
        raise TopologyError("the standard rank-order generator is specified for CP=1")
    if world_size % (tp * pp):
        raise TopologyError("world_size is not divisible by TP×PP")
    if world_size % (etp * ep * pp):
        raise TopologyError("world_size is not divisible by ETP×EP×PP")
    ddp = world_size // (tp * pp)
    edp = world_size // (etp * ep * pp)
    for n, v in (("dense_dp_degree", ddp), ("expert_dp_degree", edp)):
        if not _pow2(v):
            raise TopologyError(f"{n}={v!r} must be a positive power of two")
    dense_c, expert_c = {}, {}
    for p in range(pp):
        for d in range(ddp):
            for t in range(tp):
                dense_c[t + tp * (d + ddp * p)] = {"tp": t, "dp": d, "pp": p}
        for d in range(edp):
            for e in range(ep):
                for t in range(etp):
                    expert_c[t + etp * (e + ep * (d + edp * p))] = {"etp": t, "ep": e, "edp": d, "pp": p}
    execution = {"TP": _vary(dense_c, "tp"), "PP": _vary(dense_c, "pp"), "CP": [[r] for r in range(world_size)],
                 "EP": _vary(expert_c, "ep"), "ETP": _vary(expert_c, "etp")}
    res = analyze_topology(world_size, _vary(dense_c, "dp"), _vary(expert_c, "edp"), execution, rank_to_node)
    ref = min(ddp, edp)
    res.update(layout="power2_standard", dimensions={"tp": tp, "pp": pp, "ep": ep, "etp": etp, "cp": cp},
               degrees={"dense_dp": ddp, "expert_dp": edp}, min_dp_reference=ref)
    ok = res["candidate_replica_count"] == ref
    res["checks"]["generated_min_dp_reference_matches"] = {"pass": ok, "actual": res["candidate_replica_count"],
                                                           "reference": ref}
    if not ok:
        res["rejections"].append("coordinate-derived replica count differs from min dense/expert DP reference")
    res["valid"] = all(c["pass"] for c in res["checks"].values())
    return res


def _swap(rank: int, a: int, b: int) -> int:
    x = ((rank >> a) ^ (rank >> b)) & 1
    return rank ^ (x << a) ^ (x << b)


def make_vendor_layout(layout, rank_to_node=None) -> dict:
    """The measured 16-rank TP2/PP2/EP2/ETP2 layouts: ``legacy`` (replica on bit 2,
    PP on bit 3) or ``node_local_pp`` (bits swapped: each node holds a replica)."""
    if layout not in ("legacy", "node_local_pp"):
        raise TopologyError("layout must be 'legacy' or 'node_local_pp'")
    g = make_power2_layout(16, tp=2, pp=2, ep=2, etp=2, cp=1)["groups"]
    f = (lambda grp: sorted(_swap(r, 2, 3) for r in grp)) if layout == "node_local_pp" else (lambda grp: list(grp))
    dense = [f(x) for x in g["dense_dp"]]
    expert = [f(x) for x in g["expert_dp"]]
    execution = {n: [f(x) for x in gs] for n, gs in g["execution"].items()}
    res = analyze_topology(16, dense, expert, execution,
                           rank_to_node if rank_to_node is not None else {r: r // 8 for r in range(16)})
    res["layout"] = layout
    res["dimensions"] = {"tp": 2, "pp": 2, "ep": 2, "etp": 2, "cp": 1}
    return res


def box_layout(n_gpus: int, replicas: int = 2, tp: int = 1, pp: int = 1) -> dict:
    """The single-box layouts of this framework: ``replicas`` DP replicas of
    ``tp x pp`` GPUs each, experts split over the TP pair (EP = TP, ETP = 1).
    Rank = replica * (tp*pp) + stage * tp + tp_rank."""
    per = tp * pp
    if n_gpus != replicas * per:
        raise TopologyError(f"{n_gpus} GPUs != {replicas} replicas x {tp} TP x {pp} PP")
    coords = {r * per + s * tp + t: {"rep": r, "pp": s, "tp": t} for r in range(replicas) for s in range(pp)
              for t in range(tp)}
    dense_dp = _vary(coords, "rep")
    execution = {"TP": _vary(coords, "tp"), "PP": _vary(coords, "pp"), "EP": _vary(coords, "tp"),
                 "ETP": [[r] for r in range(n_gpus)]}
    res = analyze_topology(n_gpus, dense_dp, dense_dp, execution, {r: 0 for r in range(n_gpus)})
    res["layout"] = f"box_{replicas}x(tp{tp},pp{pp})"
    res["dimensions"] = {"replicas": replicas, "tp": tp, "pp": pp, "ep": tp, "etp": 1}
    return res
