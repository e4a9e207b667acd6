import json

import pytest

from flextensor_b200.config import OffloadConfig, load_config, load_config_from_env, load_config_from_file


def test_defaults_match_reference_schema():
    c = OffloadConfig()
    assert list(OffloadConfig.model_fields) == [
        "enabled", "gpu_device", "pinned_memory", "pinned_memory_mode", "shm_enabled", "shm_namespace",
        "shm_wait_timeout", "discovery_iters", "skip_discovery", "profiling_iters", "external_compile",
        "transfer_budget_scale", "transfer_mode", "num_blocks", "min_blocks", "max_gpu_mem_fraction",
        "profile_storage_dir", "profile_read_only", "load_strategy", "enable_instrumentation",
        "instrumentation_output_dir", "offload_timing", "piecewise_prefetch", "include_patterns", "exclude_patterns",
        "enable_diagnostics", "profile_mode",
        # beyond the reference schema
        "hold_device_weights"]
    assert (c.enabled, c.gpu_device, c.pinned_memory, c.pinned_memory_mode) == (True, 0, True, "torch")
    assert (c.shm_enabled, c.shm_namespace, c.shm_wait_timeout) == (False, None, 0.0)
    assert (c.discovery_iters, c.skip_discovery, c.profiling_iters, c.external_compile) == (1, False, 10, False)
    assert (c.transfer_budget_scale, c.transfer_mode, c.num_blocks, c.min_blocks) == (
        1.0, "allocation_block_transfer", 4, 4)
    assert c.max_gpu_mem_fraction is None and c.profile_storage_dir is None and not c.profile_read_only
    assert c.load_strategy is None and not c.enable_instrumentation
    assert c.instrumentation_output_dir == ".flextensor/instrumentation"
    assert (c.offload_timing, c.piecewise_prefetch) == ("off", "warn")
    assert c.include_patterns == ["*"] and c.exclude_patterns == []
    assert not c.enable_diagnostics and c.profile_mode == "view"
    assert c.hold_device_weights


@pytest.mark.parametrize("kw", [dict(num_blocks=2, min_blocks=3), dict(shm_enabled=True),
                                dict(profile_mode="torch_function"), dict(external_compile=True, transfer_mode="strategy"),
                                dict(offload_timing="eager", transfer_mode="strategy"), dict(warmup_iters=2),
                                dict(include_patterns=["clas:Foo"]), dict(include_patterns=[""]),
                                dict(include_patterns=[3]), dict(max_gpu_mem_fraction=1.5), dict(num_blocks=1)])
def test_invalid(kw):
    with pytest.raises(ValueError):
        OffloadConfig(**kw)


def test_pattern_normalisation():
    c = OffloadConfig(include_patterns=["  class: Linear ", "name: layers.* "])
    assert c.include_patterns == ["class:Linear", "name:layers.*"]


def test_env_precedence(monkeypatch, tmp_path):
    monkeypatch.setenv("FT_PROFILING_ITERS", "3")
    monkeypatch.setenv("FT_INCLUDE_PATTERNS", "a.*, b")
    c = load_config_from_env()
    assert c.enabled is False and c.profiling_iters == 3 and c.include_patterns == ["a.*", "b"]
    f = tmp_path / "c.json"
    f.write_text(json.dumps({"profiling_iters": 7, "num_blocks": 6, "enabled": True}))
    c = load_config(f)
    assert c.profiling_iters == 3 and c.num_blocks == 6 and c.enabled
    c = load_config(f, profiling_iters=9)
    assert c.profiling_iters == 9


def test_env_unknown_var_has_hint(monkeypatch):
    monkeypatch.setenv("FT_PROFILNG_ITERS", "3")
    with pytest.raises(ValueError, match="Did you mean: FT_PROFILING_ITERS"):
        load_config_from_env()


def test_file_formats(tmp_path):
    ini = tmp_path / "c.ini"
    ini.write_text("[flextensor]\nenabled = yes\nnum_blocks = 5\ninclude_patterns = blocks.*, head\n")
    c = load_config_from_file(ini)
    assert c.enabled and c.num_blocks == 5 and c.include_patterns == ["blocks.*", "head"]
    y = tmp_path / "c.yaml"
    y.write_text("enabled: true\nmax_gpu_mem_fraction: 0.5\n")
    assert load_config_from_file(y).max_gpu_mem_fraction == 0.5
    with pytest.raises(ValueError):
        load_config_from_file(tmp_path / "c.txt") if (tmp_path / "c.txt").write_text("x") else None
    with pytest.raises(FileNotFoundError):
        load_config_from_file(tmp_path / "missing.json")


def test_removed_field_in_file(tmp_path):
    f = tmp_path / "c.json"
    f.write_text(json.dumps({"warmup_iters": 2}))
    with pytest.raises(ValueError, match="discovery_iters"):
        load_config_from_file(f)


def test_model_copy_revalidates():
    c = OffloadConfig()
    with pytest.raises(ValueError):
        c.model_copy(update={"num_blocks": 1})
    d = c.model_copy(update={"num_blocks": 6})
    assert d.num_blocks == 6 and "num_blocks" in d.model_fields_set
