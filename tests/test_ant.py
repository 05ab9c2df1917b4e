"""Ant residency planner (host logic of the CUDA backend's VRAM tier),
checked against the reference planner's own unit tests (`src/ant.rs:802-866`)
restated, plus the properties of its greedy fill (`ant.rs:655-710`)."""

from cheetah_b200.ant import AntUnit, layer_residency_summary, plan_residency


def unit(uid, size, layer=0):
    return AntUnit(uid, size, layer)


def test_default_settings_plan_everything_into_vram():
    # ant.rs:803-813
    plan = plan_residency([unit("model.layers.0.mlp.gate_proj", 1024), unit("model.layers.0.mlp.up_proj", 1024)])
    assert plan == {"model.layers.0.mlp.gate_proj": "vram", "model.layers.0.mlp.up_proj": "vram"}


def test_layers_fill_in_numeric_order_and_the_boundary_layer_is_partial():
    # ant.rs:815-866
    units = [unit("model.layers.10.mlp.gate_proj", 600, 10), unit("model.layers.2.mlp.up_proj", 600, 2),
             unit("model.layers.2.mlp.gate_proj", 600, 2), unit("model.layers.10.mlp.up_proj", 600, 10),
             unit("model.layers.1.mlp.up_proj", 600, 1)]
    plan = plan_residency(units, vram_pool_bytes=1800, ram_budget_bytes=10_000)
    assert plan["model.layers.1.mlp.up_proj"] == "vram"
    assert plan["model.layers.2.mlp.gate_proj"] == "vram"
    assert plan["model.layers.2.mlp.up_proj"] == "vram"
    assert plan["model.layers.10.mlp.gate_proj"] == "ram"
    assert plan["model.layers.10.mlp.up_proj"] == "ram"
    summary = {e.layer_id: e for e in layer_residency_summary(units, plan)}
    assert summary[1].state() == "full_vram"
    assert summary[2].state() == "full_vram"
    assert summary[10].state() == "full_ram"
    plan = plan_residency(units, vram_pool_bytes=1500, ram_budget_bytes=10_000)
    assert plan["model.layers.1.mlp.up_proj"] == "vram"
    assert plan["model.layers.2.mlp.gate_proj"] == "vram"
    assert plan["model.layers.2.mlp.up_proj"] == "ram"
    layer2 = {e.layer_id: e for e in layer_residency_summary(units, plan)}[2]
    assert layer2.state() == "partial"
    assert (layer2.vram_units, layer2.vram_bytes, layer2.ram_units, layer2.ram_bytes) == (1, 600, 1, 600)


def test_pinned_units_go_first_and_do_not_count_against_the_pool():
    units = [unit("a", 500, 0), unit("b", 500, 1), unit("head", 900, 5)]
    plan = plan_residency(units, vram_pool_bytes=1000, ram_budget_bytes=500, resident_units=["head"])
    assert plan == {"head": "vram", "a": "vram", "b": "vram"}


def test_oversized_units_go_to_disk_and_ram_overflows_to_disk():
    units = [unit("big", 5000, 0), unit("x", 600, 1), unit("y", 600, 2), unit("z", 600, 3)]
    plan = plan_residency(units, vram_pool_bytes=1000, ram_budget_bytes=600)
    assert plan == {"big": "disk", "x": "vram", "y": "ram", "z": "disk"}


def test_disabled_ant_plans_nothing():
    assert plan_residency([unit("a", 1)], enabled=False) == {}


def test_prepared_model_plan_splits_at_a_layer(tiny_prepared):
    from cheetah_b200.ant import units_of
    from cheetah_b200.prepared import PreparedModel

    units = units_of(PreparedModel(tiny_prepared))
    layer0 = sum(u.bytes for u in units if u.layer_id == 0)
    plan = plan_residency(units, vram_pool_bytes=layer0, ram_budget_bytes=1 << 40)
    tiers = {e.layer_id: e.state() for e in layer_residency_summary(units, plan)}
    assert tiers[0] == "full_vram" and tiers[1] == "full_ram"
