"""Topology planner: standard and measured layouts, validation errors, and
this framework's single-box layouts."""
import pytest

from shift_b200.parallel.topology import (TABLE_4_2, TopologyError, analyze_topology, box_layout,
                                          make_power2_layout, make_vendor_layout)


@pytest.mark.parametrize("name,expected", [("A", 2), ("B", 2), ("C", 4), ("D", 8)])
def test_table_layouts_replica_counts_and_sources(name, expected):
    plan = make_power2_layout(16, cp=1, **TABLE_4_2[name])
    assert plan["valid"], plan["rejections"]
    assert plan["candidate_replica_count"] == expected == plan["min_dp_reference"]
    assert {r["size"] for r in plan["replicas"]} == {16 // expected}
    for key in ("roles_one_each", "groups_inside_replicas", "single_recovery_source",
                "replicas_equal_min_dp_degree"):
        assert plan["checks"][key]["pass"], key
    for rank, sources in plan["recovery_sources"].items():
        assert len(sources) == expected - 1
        assert all(isinstance(s, int) for s in sources.values())


def test_vendor_layouts_node_failure_survival():
    legacy = make_vendor_layout("legacy")
    local = make_vendor_layout("node_local_pp")
    assert legacy["valid"] and local["valid"]
    assert legacy["candidate_replica_count"] == local["candidate_replica_count"] == 2
    assert legacy["survivable_replicas_by_node_failure"] == {0: [], 1: []}
    assert local["survivable_replicas_by_node_failure"] == {0: [1], 1: [0]}
    assert [r["ranks"] for r in local["replicas"]] == [list(range(8)), list(range(8, 16))]
    assert all(v == 0 for v in local["execution_groups_crossing_nodes"].values())
    assert legacy["execution_groups_crossing_nodes"]["PP"] > 0


def test_overlapping_group_rejected():
    g = make_power2_layout(16, tp=2, pp=2, ep=4, etp=1)["groups"]
    bad = [[0, 1], [1, 2]] + [[r] for r in range(3, 16)]
    with pytest.raises(TopologyError, match="rank 1 is in both group #0 and group #1"):
        analyze_topology(16, g["dense_dp"], g["expert_dp"], {**g["execution"], "TP": bad})


def test_missing_dense_expert_source_reported():
    g = make_power2_layout(16, tp=2, pp=2, ep=4, etp=1)["groups"]
    res = analyze_topology(16, g["dense_dp"], [[r] for r in range(16)], g["execution"])
    assert res["candidate_replica_count"] == 2 and not res["valid"]
    assert not res["checks"]["single_recovery_source"]["pass"]
    assert "missing or ambiguous source" in " ".join(res["rejections"])


def test_non_power_of_two():
    res = analyze_topology(6, [[0, 1, 2], [3, 4, 5]], [[0, 1, 2], [3, 4, 5]], {"TP": [list(range(6))]})
    assert res["candidate_replica_count"] == 1 and not res["valid"]
    assert res["metrics"]["dense_dp_group_sizes"] == [3, 3]
    with pytest.raises(TopologyError, match="world_size=12.*powers of two"):
        make_power2_layout(12, tp=2, pp=2, ep=2, etp=1)


def test_fused_execution_dependency_merges_replicas():
    g = make_power2_layout(16, tp=2, pp=2, ep=4, etp=1)["groups"]
    res = analyze_topology(16, g["dense_dp"], g["expert_dp"], {**g["execution"], "FUSED": [list(range(16))]})
    assert res["candidate_replica_count"] == 1
    assert res["checks"]["groups_inside_replicas"]["pass"]
    assert not res["checks"]["single_recovery_source"]["pass"]


def test_dp_family_names_rejected_and_infeasible_layout():
    with pytest.raises(TopologyError, match="replicates state"):
        analyze_topology(2, [[0, 1]], [[0, 1]], {"DP": [[0], [1]]})
    # EP2 x ETP2 x PP2 needs 8 ranks per replica: a 4-GPU replica cannot hold it
    with pytest.raises(TopologyError, match="ETP×EP×PP blocks"):
        make_power2_layout(4, tp=2, pp=2, ep=2, etp=2)


@pytest.mark.parametrize("n,tp,pp", [(2, 1, 1), (4, 2, 1), (8, 2, 2), (8, 1, 1)])
def test_box_layouts(n, tp, pp):
    reps = n // (tp * pp)
    plan = box_layout(n, replicas=reps, tp=tp, pp=pp)
    assert plan["valid"], plan["rejections"]
    assert plan["candidate_replica_count"] == reps
    # every rank recovers from the same position of every other replica
    for rank, src in plan["recovery_sources"].items():
        for other, s in src.items():
            assert s % (tp * pp) == rank % (tp * pp)


@pytest.mark.parametrize("groups,msg", [
    (None, "no groups given"),
    (5, "expected a list of rank lists"),
    ([], "the list of groups is empty"),
    ([[0, 1], []], "group #1 has no ranks"),
    ([[0, 1], [2, 9]], "names 9, which is not a rank"),
    ([[0, 0], [1, 2, 3]], "rank 0 is listed twice"),
    ([[0, 1], [2]], r"ranks \[3\] belong to no group"),
    ([[0, True], [2, 3]], "names True"),
])
def test_malformed_groups_rejected(groups, msg):
    with pytest.raises(TopologyError, match=msg):
        analyze_topology(4, groups, [[0, 1], [2, 3]], {"TP": [[0], [1], [2], [3]]})


def test_rank_to_node_validation_and_label_propagation_order():
    ex = {"TP": [[0, 3], [1], [2]], "PP": [[3, 2], [0], [1]]}   # 0-3-2 chained through two families
    res = analyze_topology(4, [[0, 1], [2], [3]], [[0, 1], [2], [3]], ex, rank_to_node=[0, 0, 1, 1])
    assert [r["ranks"] for r in res["replicas"]] == [[0, 2, 3], [1]]
    assert res["survivable_replicas_by_node_failure"] == {0: [], 1: [1]}
    with pytest.raises(TopologyError, match="lists 3 nodes for 4 ranks"):
        analyze_topology(4, [[0, 1, 2, 3]], [[0, 1, 2, 3]], {"TP": [[0], [1], [2], [3]]}, rank_to_node=[0, 0, 1])
    with pytest.raises(TopologyError, match=r"without a node \[3\]"):
        analyze_topology(4, [[0, 1, 2, 3]], [[0, 1, 2, 3]], {"TP": [[0], [1], [2], [3]]},
                         rank_to_node={0: 0, 1: 0, 2: 1})
