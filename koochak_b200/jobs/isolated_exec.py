"""Run a Python target (``-m mod``, ``-c code`` or a script) after adding explicit import roots.

(reference: koochak/jobs/isolated_exec.py:22-77)

    python -I -m koochak_b200.jobs.isolated_exec '["/src"]' -- -m pkg.train --config x.yaml

The runner starts workloads with ``python -I`` (no user site, no PYTHONPATH);
the profile's PYTHONPATH entries arrive here as an explicit JSON list
instead. A ``CheckpointArtifactAckTimeout`` escaping the target becomes its
own exit code (76) with a ``checkpoint_safe_retry`` note, so a scheduler can
retry the run with auto-resume rather than treat it as an application error.
"""

from __future__ import annotations

import json
import runpy
import sys
from pathlib import Path
from typing import List, Tuple

__all__ = ["main"]


def _split_target(args: List[str]) -> Tuple[str, str, List[str]]:
    for i, a in enumerate(args):
        if a in ("-m", "-c"):
            if i + 1 >= len(args):
                raise ValueError(f"{a} requires a target")
            return a, args[i + 1], args[i + 2:]
        if not a.startswith("-"):
            return "script", a, args[i + 1:]
    raise ValueError("isolated Python child has no module, script, or command target")


def main(argv: List[str] | None = None) -> int:
    args = sys.argv[1:] if argv is None else list(argv)
    if "--" not in args:
        raise SystemExit("isolated_exec requires '--' before the original Python arguments")
    sep = args.index("--")
    try:
        roots = json.loads(args[0])
        if not isinstance(roots, list) or not all(isinstance(r, str) for r in roots):
            raise ValueError("import roots must be a list of strings")
        mode, target, rest = _split_target(args[sep + 1:])
    except (IndexError, TypeError, ValueError) as exc:
        raise SystemExit(f"invalid isolated Python invocation: {exc}") from exc
    for r in reversed(roots):
        sys.path.insert(0, r)
    try:
        if mode == "-m":
            sys.argv = [target, *rest]
            runpy.run_module(target, run_name="__main__", alter_sys=True)
        elif mode == "-c":
            sys.argv = ["-c", *rest]
            ns = {"__name__": "__main__", "__file__": "<string>"}
            exec(compile(target, "<string>", "exec"), ns, ns)  # noqa: S102 - the declared workload
        else:
            sys.argv = [str(Path(target)), *rest]
            runpy.run_path(str(Path(target)), run_name="__main__")
    except Exception as exc:
        code = getattr(exc, "exit_code", None)
        if getattr(exc, "reason", None) == "checkpoint_ack_timeout" and type(code) is int:
            print(json.dumps({"kind": "checkpoint_safe_retry", "reason": "checkpoint_ack_timeout",
                              "checkpoint_path": getattr(exc, "checkpoint_path", None),
                              "event_id": getattr(exc, "event_id", None)}, sort_keys=True), file=sys.stderr)
            return code
        raise
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
