"""Host-side rules of the graphed step (no GPU): when an update may go through the graph."""

from __future__ import annotations

import torch

from koochak_b200.runtime.graphed_step import GraphedStep, _signature
from koochak_b200.runtime.settings import LoopSettings


def test_signature_needs_a_mapping_of_tensors():
    assert _signature({"idx": torch.zeros(2, 3, dtype=torch.long)}) is not None
    assert _signature([torch.zeros(2)]) is None
    assert _signature({"idx": torch.zeros(2), "note": "x"}) is None
    a = _signature({"b": torch.zeros(2), "a": torch.zeros(3)})
    b = _signature({"a": torch.zeros(3), "b": torch.zeros(2)})
    assert a == b  # key order does not matter
    assert a != _signature({"a": torch.zeros(4), "b": torch.zeros(2)})


def test_capture_waits_for_the_eager_warm_up():
    g = GraphedStep(torch.nn.Linear(2, 2), warmup=2)
    batch = {"x": torch.zeros(4, 2)}
    assert not g.wants(batch)
    g.note_eager()
    assert not g.wants(batch)
    g.note_eager()
    assert g.wants(batch)
    assert not g.wants([torch.zeros(1)])
    g.disabled = True
    assert not g.wants(batch)


def test_settings_keys():
    s = LoopSettings.from_cfg({"cuda_graph_step": True, "cuda_graph_warmup": 5})
    assert s.cuda_graph_step is True and s.cuda_graph_warmup == 5
    assert LoopSettings.from_cfg({}).cuda_graph_step is False
