"""Binding-time annotations: the staging surface the residual path sits behind.

Same names and behaviour as the reference's ``stageml.annotations``
(stageml/annotations.py:10-74): a two-point lattice where ``stage0`` values are
known at deploy time (folded ahead of time, e.g. the LoRA merge W + s*B*A) and
``stage1`` values arrive per request (the residual program: routing, expert
GEMMs, dynamic LoRA). ``compile_staged`` reads the annotations of a function's
parameters into a staging environment; unannotated parameters are stage1.
No compute happens here.
"""

from __future__ import annotations

import inspect
from dataclasses import dataclass
from typing import Callable


@dataclass(frozen=True)
class BindingTime:
    level: int  # 0 = static (deploy time), 1 = dynamic (request time)
    name: str

    def __repr__(self) -> str:
        return self.name

    def join(self, other: "BindingTime") -> "BindingTime":
        """Least upper bound: dynamic if either side is dynamic."""
        return stage1 if (self.level == 1 or other.level == 1) else stage0


stage0 = BindingTime(level=0, name="stage0")
stage1 = BindingTime(level=1, name="stage1")


def build_staging_env(fn: Callable) -> dict[str, BindingTime]:
    """Map each parameter of ``fn`` to its binding time (annotation or stage1)."""
    env: dict[str, BindingTime] = {}
    for name, ann in getattr(fn, "__annotations__", {}).items():
        if name == "return":
            continue
        env[name] = ann if isinstance(ann, BindingTime) else stage1
    for name in inspect.signature(fn).parameters:
        env.setdefault(name, stage1)
    return env


def compile_staged(fn: Callable) -> Callable:
    """Attach the staging environment to ``fn`` and give it ``analyze``/``compile`` hooks."""
    gamma = build_staging_env(fn)
    fn._gamma = gamma
    fn._staged = True
    fn._compiled_fn = None

    def analyze() -> None:
        rule = "-" * 50
        print(f"\n{rule}\nStageML Staging Analysis: {fn.__name__}\n{rule}")
        print(f"{'Parameter':<20} {'Binding Time':<15} Meaning\n{rule}")
        for name, bt in gamma.items():
            meaning = "compile-time static" if bt == stage0 else "runtime dynamic"
            print(f"  {name:<18} {str(bt):<15} {meaning}")
        print(rule)

    def compile() -> Callable:
        print(f"[StageML] Compiling {fn.__name__}...")
        print(f"  Staging environment: {gamma}")
        return fn

    fn.analyze = analyze
    fn.compile = compile
    return fn


__all__ = ["BindingTime", "stage0", "stage1", "build_staging_env", "compile_staged"]
