"""Preparing one launch and handing it to a scheduler.

``prepared_run()`` builds the immutable launch (environment profile, argv,
config snapshot) once; the same object can then be staged and run locally by
the isolated runner, or submitted through one of the optional scheduler
adapters. Paths are placeholders for a shared filesystem.
"""

from __future__ import annotations

from koochak_b200.jobs import Preemptible, load_environment_profile, prepare_run, stage_run


def prepared_run(preemptible: bool = False):
    return prepare_run(
        name="mnist-example",
        profile=load_environment_profile("examples/jobs/environment.yaml"),
        python_args=["-m", "koochak_b200.cli.train", "--config", "{config}"],
        cwd="/shared/project/repo",
        run_dir="/shared/project/runs/mnist-example",
        base_config="examples/mnist/config.yaml",
        preemptible=Preemptible() if preemptible else False,
    )


def stage_locally() -> str:
    """Write launch.json, the config snapshot and the runner entry under run_dir."""

    prepared = prepared_run()
    stage_run(prepared)
    return prepared.run_dir


def submit_to_scruffy(root: str, resources: object, request_id: str, project_id: str) -> dict:
    """Submit through the Scruffy adapter (needs the optional ``scruffy`` client installed)."""

    from koochak_b200.jobs import submit_scruffy

    return submit_scruffy(prepared_run(), root=root, resources=resources, request_id=request_id,
                          project_id=project_id)


if __name__ == "__main__":
    run = prepared_run()
    print(run.runner_argv())
