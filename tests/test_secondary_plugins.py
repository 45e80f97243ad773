"""Secondary plugins: the default registry holds the engine's real components,
with the reference's register / activate / execute / deactivate lifecycle."""
from mod_b200.api import SecondaryPlugin, SecondaryPluginManager, SecondaryPluginType as T, get_secondary_plugin_manager
from mod_b200.config import get_preset


def test_defaults_cover_every_kind():
    m = get_secondary_plugin_manager()
    listing = m.list()
    assert all(listing[k.value] for k in T), listing
    assert set(listing["distributed_execution"]) == {"fused-nvlink", "nvls", "nccl"}


def test_activate_execute_deactivate():
    m = SecondaryPluginManager(defaults=True)
    assert m.execute_plugin(T.SHARDING) is None                  # not active yet
    assert m.activate_plugin(T.SHARDING)
    plan = m.execute_plugin(T.SHARDING, get_preset("qwen3-30b-a3b"), 8)
    assert plan.ep == 8 and plan.fits
    assert m.activate_plugin(T.MEMORY_MANAGER, device="cpu")
    assert isinstance(m.execute_plugin(T.MEMORY_MANAGER), dict)
    assert m.activate_plugin(T.DISTRIBUTED_EXECUTION, "nccl", parallelism="ep")
    assert m.execute_plugin(T.DISTRIBUTED_EXECUTION).__name__ == "NcclEPMoE"
    assert m.activate_plugin(T.DISTRIBUTED_EXECUTION, "nvls", parallelism="tp")
    assert m.execute_plugin(T.DISTRIBUTED_EXECUTION).__name__ == "NvlsTP"
    assert m.deactivate_plugin(T.SHARDING) and m.execute_plugin(T.SHARDING) is None


def test_budget_plugin_rejects_overrun():
    import pytest

    from mod_b200.runtime.memory import OutOfBudget

    m = SecondaryPluginManager(defaults=True)
    assert m.activate_plugin(T.SECURITY, device="cpu")
    m.get_plugin(T.SECURITY).instance.define("kv", 100)
    m.execute_plugin(T.SECURITY, "kv", 60)
    with pytest.raises(OutOfBudget):
        m.execute_plugin(T.SECURITY, "kv", 60)


def test_failed_initialisation_is_reported():
    m = SecondaryPluginManager()

    def boom(**kw):
        raise RuntimeError("no device")

    m.register_plugin(T.COMPRESSION, SecondaryPlugin("bad", boom))
    assert not m.activate_plugin(T.COMPRESSION, "bad")
