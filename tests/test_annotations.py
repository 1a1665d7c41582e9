"""Binding-time surface (same behaviour as the reference's stageml.annotations and its tests)."""

from stageml_b200 import BindingTime, compile_staged, stage0, stage1
from stageml_b200.annotations import build_staging_env


def test_lattice_join():
    assert stage0.join(stage0) == stage0
    assert stage0.join(stage1) == stage1
    assert stage1.join(stage0) == stage1
    assert stage1.join(stage1) == stage1
    assert repr(stage0) == "stage0" and repr(stage1) == "stage1"
    assert BindingTime(0, "stage0") == stage0


def test_staging_env_defaults_to_stage1():
    def f(x, W: stage0, b: stage1, c: int) -> stage1:
        return x

    env = build_staging_env(f)
    assert env == {"x": stage1, "W": stage0, "b": stage1, "c": stage1}


def test_compile_staged_decorator(capsys):
    @compile_staged
    def layer(x, W: stage0, A: stage0, B: stage0):
        return x

    assert layer._staged and layer._gamma["W"] == stage0 and layer._gamma["x"] == stage1
    assert layer.compile() is layer
    layer.analyze()
    out = capsys.readouterr().out
    assert "compile-time static" in out and "runtime dynamic" in out
