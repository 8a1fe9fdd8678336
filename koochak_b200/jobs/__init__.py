"""Reproducible, isolated launches of training runs (no PyTorch import).

(reference: koochak/jobs/__init__.py)

Public names resolve lazily, so ``import koochak_b200.jobs`` costs only the
standard library; the runner reads its JSON manifest the same way.
"""

from importlib import import_module

_WHERE = {
    "ConfigPatch": ".manifest", "Preemptible": ".manifest", "PreparedRun": ".manifest",
    "materialize_config": ".manifest", "prepare_run": ".manifest", "stage_run": ".manifest",
    "EnvironmentProfile": ".profile", "load_environment_profile": ".profile",
    "PreparedTask": ".workflow", "PreparedWorkflow": ".workflow",
    "DeclaredOutput": "..storage.artifact",
    "submit_pazuzu": ".backends", "submit_scruffy": ".backends", "submit_scruffy_workflow": ".backends",
}
__all__ = sorted(_WHERE)


def __getattr__(name):
    if name not in _WHERE:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(import_module(_WHERE[name], __name__), name)
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(__all__))
