"""koochak_b200: a function-first training runtime for NVIDIA B200 (sm_100a).

Public entry points mirror jamaliki/koochak: ``training_loop``, the config
helpers, the Muon/AdamW optimizer builders, EMA, checkpoint publication and
the evacuation controller. Hot paths run on hand-written sm_100a kernels
(``koochak_b200.ops``) when tensors live on a CUDA device.
"""

from .interruption import (CHECKPOINT_ACK_TIMEOUT_EXIT_CODE, EVACUATION_EXIT_CODE, OOM_RESTART_EXIT_CODE,
                           EvacuationController, install_evacuation_handler)

__version__ = "0.1.0"

__all__ = ["CHECKPOINT_ACK_TIMEOUT_EXIT_CODE", "EVACUATION_EXIT_CODE", "OOM_RESTART_EXIT_CODE",
           "EvacuationController", "install_evacuation_handler", "training_loop"]


def __getattr__(name):
    if name == "training_loop":
        from .loop import training_loop

        return training_loop
    raise AttributeError(name)
