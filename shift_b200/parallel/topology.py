"""Topology planner: which ranks form a recoverable replica, and where each
rank's state can be recovered from.

A job is described by its rank groups: dense data-parallel groups, expert
data-parallel groups, and any number of named execution families (TP, PP,
CP, EP, ETP, ...).  Ranks tied together by an execution family compute in
lock-step, so they fail and are replaced as a unit: the connected
components of all execution groups are the candidate replicas.  A plan is
usable for live recovery when

* there are two or more replicas, all of one size;
* every replica holds each local role (the rank's position inside each of
  its execution groups) exactly once, and all replicas hold the same roles;
* no execution group reaches into two replicas;
* every rank has, in every other replica, exactly one rank of the same role
  that shares both its dense-DP and its expert-DP group (so dense and expert
  state can be fetched from a single peer).

Given a rank -> node map the planner also says which replicas survive the
loss of each node and how many execution groups span nodes.

Behaviour and result keys follow shift_full/topology.py:102-285 (analysis),
:304-367 (power-of-two layouts) and :375-402 (the measured 16-rank layouts).
The rank orders are Megatron's conventions -- dense
``tp + TP*(dp + DP*pp)``, expert ``etp + ETP*(ep + EP*(edp + EDP*pp))`` -- and
``node_local_pp`` exchanges rank bits 2 and 3 so each 8-rank node holds one
whole replica.  ``box_layout`` adds the layouts this framework runs on one
8-GPU box.
"""
from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass

# Table 4.2 of the SHIFT paper: per-replica parallel sizes of four 16-rank layouts.
TABLE_4_2 = {
    "A": {"tp": 2, "pp": 2, "ep": 4, "etp": 1},
    "B": {"tp": 4, "pp": 2, "ep": 2, "etp": 1},
    "C": {"tp": 2, "pp": 1, "ep": 4, "etp": 1},
    "D": {"tp": 2, "pp": 1, "ep": 2, "etp": 1},
}

# families that replicate state instead of splitting work; they never bind ranks into one replica
_REPLICATING_FAMILIES = frozenset({"DP", "DENSE_DP", "EXPERT_DP", "EDP"})


class TopologyError(ValueError):
    """Malformed topology input or an unsupported generated layout."""


def _is_int(x) -> bool:
    return type(x) is int          # bool is a subclass of int and is not a rank


def _power_of_two(x) -> bool:
    return _is_int(x) and x > 0 and x & (x - 1) == 0


# ---------------------------------------------------------------------- groups
@dataclass(frozen=True)
class Partition:
    """Disjoint rank groups that together cover ranks 0..world-1, in a
    canonical order (each group ascending, groups ordered by their ranks)."""

    label: str
    groups: tuple
    owner: tuple            # owner[rank] -> index into groups

    @classmethod
    def build(cls, label: str, groups, world: int) -> "Partition":
        if groups is None:
            raise TopologyError(f"{label}: no groups given")
        try:
            members = [tuple(g) for g in groups]
        except TypeError as e:
            raise TopologyError(f"{label}: expected a list of rank lists, got {type(groups).__name__}") from e
        if not members:
            raise TopologyError(f"{label}: the list of groups is empty")
        where = [-1] * world
        for gi, g in enumerate(members):
            if not g:
                raise TopologyError(f"{label}: group #{gi} has no ranks")
            for r in g:
                if not _is_int(r) or not 0 <= r < world:
                    raise TopologyError(f"{label}: group #{gi} names {r!r}, which is not a rank in [0, {world})")
                if where[r] == gi:
                    raise TopologyError(f"{label}: rank {r} is listed twice in group #{gi}")
                if where[r] >= 0:
                    raise TopologyError(f"{label}: rank {r} is in both group #{where[r]} and group #{gi}")
                where[r] = gi
        orphans = [r for r in range(world) if where[r] < 0]
        if orphans:
            raise TopologyError(f"{label}: ranks {orphans} belong to no group")
        canon = tuple(sorted(tuple(sorted(g)) for g in members))
        owner = [0] * world
        for gi, g in enumerate(canon):
            for r in g:
                owner[r] = gi
        return cls(label, canon, tuple(owner))

    def of(self, rank: int) -> tuple:
        return self.groups[self.owner[rank]]

    def sizes(self) -> list:
        return sorted(len(g) for g in self.groups)

    def as_lists(self) -> list:
        return [list(g) for g in self.groups]


def _components(world: int, families: dict) -> list:
    """Connected components of the union of all execution groups, found by
    minimum-label propagation: every group adopts the smallest label among
    its ranks until nothing changes.  Components are returned ascending by
    their smallest rank."""
    label = list(range(world))
    moved = True
    while moved:
        moved = False
        for part in families.values():
            for g in part.groups:
                low = min(label[r] for r in g)
                for r in g:
                    if label[r] != low:
                        label[r] = low
                        moved = True
    comp: dict = {}
    for r in range(world):
        comp.setdefault(label[r], []).append(r)
    return [tuple(comp[k]) for k in sorted(comp)]


def _node_map(rank_to_node, world: int) -> dict:
    if isinstance(rank_to_node, Mapping):
        nodes = dict(rank_to_node)
    elif isinstance(rank_to_node, Sequence) and not isinstance(rank_to_node, (str, bytes)):
        if len(rank_to_node) != world:
            raise TopologyError(f"rank_to_node lists {len(rank_to_node)} nodes for {world} ranks")
        nodes = dict(enumerate(rank_to_node))
    else:
        raise TopologyError("rank_to_node must map ranks to nodes (a dict, or a list indexed by rank)")
    unknown = sorted(r for r in nodes if not (_is_int(r) and 0 <= r < world))
    absent = sorted(set(range(world)) - set(nodes))
    if unknown or absent:
        raise TopologyError(f"rank_to_node does not cover exactly ranks 0..{world - 1}: "
                            f"without a node {absent}, not ranks {unknown}")
    return nodes


# ---------------------------------------------------------------------- analysis
class _Verdict:
    """Collects named checks (``{"pass": bool, ...details}``) and, for each
    failed one, a sentence saying why the plan is unusable."""

    def __init__(self):
        self.checks: dict = {}
        self.rejections: list = []

    def add(self, name: str, ok: bool, why: str, **detail):
        self.checks[name] = {"pass": bool(ok), **detail}
        if not ok:
            self.rejections.append(why)

    @property
    def valid(self) -> bool:
        return all(c["pass"] for c in self.checks.values())


def analyze_topology(world_size, dense_dp_groups, expert_dp_groups, execution_groups, rank_to_node=None) -> dict:
    if not _is_int(world_size) or world_size < 1:
        raise TopologyError(f"world_size must be a positive int, got {world_size!r}")
    W = world_size
    dense = Partition.build("dense_dp", dense_dp_groups, W)
    expert = Partition.build("expert_dp", expert_dp_groups, W)
    if not isinstance(execution_groups, Mapping) or not execution_groups:
        raise TopologyError("execution_groups must map at least one family name to its rank groups")
    fam: dict = {}
    for raw_name, groups in execution_groups.items():
        name = str(raw_name).upper()
        if name in _REPLICATING_FAMILIES:
            raise TopologyError(f"{name} replicates state (a DP family); list it as dense/expert DP, "
                                f"not as an execution family")
        if name in fam:
            raise TopologyError(f"execution family {name} is given twice (names are case-insensitive)")
        fam[name] = Partition.build(f"execution family {name}", groups, W)
    names = sorted(fam)

    replicas = _components(W, fam)
    replica_of = {r: i for i, ranks in enumerate(replicas) for r in ranks}
    position = {r: {n: fam[n].of(r).index(r) for n in names} for r in range(W)}
    role = {r: tuple(position[r][n] for n in names) for r in range(W)}
    n_rep = len(replicas)

    v = _Verdict()
    v.add("replica_count", n_rep >= 2,
          f"only {n_rep} replica found: a failed replica would have no live peer to recover from",
          actual=n_rep)
    sizes = [len(rs) for rs in replicas]
    v.add("replica_sizes_equal", len(set(sizes)) == 1, f"replicas differ in size: {sizes}", sizes=sizes)

    roles_per = [[role[r] for r in rs] for rs in replicas]
    repeats = [i for i, rl in enumerate(roles_per) if len(set(rl)) != len(rl)]
    base = set(roles_per[0]) if roles_per else set()
    differ = [i for i, rl in enumerate(roles_per) if set(rl) != base]
    v.add("roles_one_each", not repeats and not differ,
          f"replicas {sorted(set(repeats) | set(differ))} do not hold the same local roles once each",
          role_counts=[len(set(rl)) for rl in roles_per], duplicate_role_replicas=repeats)

    spanning = [{"group": n, "ranks": list(g), "replicas": sorted({replica_of[r] for r in g})}
                for n in names for g in fam[n].groups if len({replica_of[r] for r in g}) > 1]
    v.add("groups_inside_replicas", not spanning,
          f"{len(spanning)} execution group(s) reach into more than one replica", groups=spanning)

    shared = {r: sorted(set(dense.of(r)) & set(expert.of(r))) for r in range(W)}
    sources: dict = {}
    gaps = []
    for r in range(W):
        sources[r] = {}
        for other in range(n_rep):
            if other == replica_of[r]:
                continue
            found = [s for s in shared[r] if replica_of[s] == other and role[s] == role[r]]
            sources[r][other] = found[0] if len(found) == 1 else found
            if len(found) != 1:
                gaps.append({"rank": r, "target_replica": other, "candidates": found})
    v.add("single_recovery_source", not gaps and n_rep >= 2,
          f"{len({g['rank'] for g in gaps})} rank(s) lack exactly one same-role peer inside both their "
          f"dense-DP and expert-DP groups in some other replica (missing or ambiguous source)", issues=gaps)

    survivable, crossing = {}, {}
    if rank_to_node is not None:
        nodes = _node_map(rank_to_node, W)
        for node in sorted(set(nodes.values()), key=str):
            survivable[node] = [i for i, rs in enumerate(replicas) if node not in {nodes[r] for r in rs}]
        crossing = {n: sum(1 for g in fam[n].groups if len({nodes[r] for r in g}) > 1) for n in names}

    return {
        "valid": v.valid,
        "world_size": W,
        "candidate_replica_count": n_rep,
        "replicas": [{"id": i, "ranks": list(rs), "size": len(rs), "role_count": len(set(roles_per[i]))}
                     for i, rs in enumerate(replicas)],
        "rank_to_replica": replica_of,
        "rank_to_localrole": position,
        "recovery_sources": sources,
        "dense_expert_intersections": shared,
        "survivable_replicas_by_node_failure": survivable,
        "execution_groups_crossing_nodes": crossing,
        "checks": v.checks,
        "rejections": v.rejections,
        "metrics": {"dense_dp_group_sizes": dense.sizes(), "expert_dp_group_sizes": expert.sizes(),
                    "dense_expert_intersection_sizes": {r: len(s) for r, s in shared.items()},
                    "execution_group_sizes": {n: fam[n].sizes() for n in names}},
        "groups": {"dense_dp": dense.as_lists(), "expert_dp": expert.as_lists(),
                   "execution": {n: fam[n].as_lists() for n in names}},
    }


# ---------------------------------------------------------------------- generated layouts
def _decompose(rank: int, radices: list) -> list:
    """Mixed-radix digits of ``rank``, least significant first."""
    out = []
    for base in radices:
        rank, d = divmod(rank, base)
        out.append(d)
    return out


def _along(coords: dict, axis: str) -> list:
    """Rank groups whose coordinates agree on every axis except ``axis``."""
    by_rest: dict = {}
    for r in sorted(coords):
        rest = tuple(sorted((k, x) for k, x in coords[r].items() if k != axis))
        by_rest.setdefault(rest, []).append(r)
    return list(by_rest.values())


def make_power2_layout(world_size, tp, pp, ep, etp, cp=1, rank_to_node=None) -> dict:
    for name, x in (("world_size", world_size), ("tp", tp), ("pp", pp), ("ep", ep), ("etp", etp), ("cp", cp)):
        if not _power_of_two(x):
            raise TopologyError(f"{name}={x!r}: the generator handles positive powers of two only")
    if cp != 1:
        raise TopologyError(f"cp={cp}: the Megatron rank orders used here are defined without context parallelism")
    if world_size % (tp * pp):
        raise TopologyError(f"{world_size} ranks cannot hold whole TP×PP blocks of {tp * pp}")
    if world_size % (etp * ep * pp):
        raise TopologyError(f"{world_size} ranks cannot hold whole ETP×EP×PP blocks of {etp * ep * pp}")
    ddp = world_size // (tp * pp)
    edp = world_size // (etp * ep * pp)
    dense_c, expert_c = {}, {}
    for r in range(world_size):
        t, d, p = _decompose(r, [tp, ddp, pp])                  # r = t + tp*(d + ddp*p)
        dense_c[r] = {"tp": t, "dp": d, "pp": p}
        et, e, ed, p2 = _decompose(r, [etp, ep, edp, pp])       # r = et + etp*(e + ep*(ed + edp*p2))
        expert_c[r] = {"etp": et, "ep": e, "edp": ed, "pp": p2}
    execution = {"TP": _along(dense_c, "tp"), "PP": _along(dense_c, "pp"),
                 "CP": [[r] for r in range(world_size)],
                 "EP": _along(expert_c, "ep"), "ETP": _along(expert_c, "etp")}
    res = analyze_topology(world_size, _along(dense_c, "dp"), _along(expert_c, "edp"), execution, rank_to_node)
    expect = min(ddp, edp)
    res.update(layout="power2_standard", dimensions={"tp": tp, "pp": pp, "ep": ep, "etp": etp, "cp": cp},
               degrees={"dense_dp": ddp, "expert_dp": edp}, min_dp_reference=expect)
    agree = res["candidate_replica_count"] == expect
    res["checks"]["replicas_equal_min_dp_degree"] = {"pass": agree, "actual": res["candidate_replica_count"],
                                                     "reference": expect}
    if not agree:
        res["rejections"].append(f"{res['candidate_replica_count']} replicas derived from the groups, but "
                                 f"min(dense DP, expert DP) = {expect}")
    res["valid"] = all(c["pass"] for c in res["checks"].values())
    return res


def _exchange_bits_2_3(rank: int) -> int:
    b2, b3 = (rank >> 2) & 1, (rank >> 3) & 1
    return (rank & ~0b1100) | (b2 << 3) | (b3 << 2)


def make_vendor_layout(layout, rank_to_node=None) -> dict:
    """The measured 16-rank TP2/PP2/EP2/ETP2 layouts: ``legacy`` (replica on
    bit 2, PP on bit 3) or ``node_local_pp`` (the two bits exchanged, so each
    8-rank node holds one replica)."""
    if layout not in ("legacy", "node_local_pp"):
        raise TopologyError(f"unknown vendor layout {layout!r} (choose 'legacy' or 'node_local_pp')")
    base = make_power2_layout(16, tp=2, pp=2, ep=2, etp=2, cp=1)["groups"]
    if layout == "node_local_pp":
        remap = lambda grp: sorted(_exchange_bits_2_3(r) for r in grp)  # noqa: E731
    else:
        remap = lambda grp: list(grp)  # noqa: E731
    res = analyze_topology(16, [remap(g) for g in base["dense_dp"]], [remap(g) for g in base["expert_dp"]],
                           {n: [remap(g) for g in gs] for n, gs in base["execution"].items()},
                           rank_to_node if rank_to_node is not None else [r // 8 for r in range(16)])
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
    coords = {}
    for r in range(n_gpus):
        t, s, rep = _decompose(r, [tp, pp, replicas])
        coords[r] = {"rep": rep, "pp": s, "tp": t}
    dense_dp = _along(coords, "rep")
    execution = {"TP": _along(coords, "tp"), "PP": _along(coords, "pp"), "EP": _along(coords, "tp"),
                 "ETP": [[r] for r in range(n_gpus)]}
    res = analyze_topology(n_gpus, dense_dp, dense_dp, execution, [0] * n_gpus)
    res["layout"] = f"box_{replicas}x(tp{tp},pp{pp})"
    res["dimensions"] = {"replicas": replicas, "tp": tp, "pp": pp, "ep": tp, "etp": 1}
    return res
