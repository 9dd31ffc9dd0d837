"""Host metadata of the row pools (CPU): deepseekrpc_b200.cache_pool.SlotMap replays a
trace recorded from the reference's own SlotMap (tests/golden/make_golden.py), and
refuses what the reference refuses."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from deepseekrpc_b200.cache_pool import Operation, SlotMap
from deepseekrpc_b200.cuda_ops import ValidationError

TRACE = Path(__file__).resolve().parent / "golden" / "slotmap_trace.json"


# the reference's refusal messages recorded in the trace, and the reason this
# module tags the same refusal with
REFUSALS = {"one scatter batch repeats a physical cache slot": "repeat"}


def test_slot_map_replays_the_reference_trace():
    for case in json.loads(TRACE.read_text()):
        mapping = SlotMap(case["slots"], context=64, offset=case["offset"], max_mutations=16)
        mapping.reset("a" * 32, 0)
        for step in case["steps"]:
            op = Operation("a" * 32, 0, step["start"], step["rows"])
            mapping.begin(op)
            try:
                got = mapping.reserve(step["logical"], list(range(step["start"], step["start"] + step["rows"])))
                reserved, reason = [list(map(int, got[0])), list(map(int, got[1]))], None
            except ValidationError as e:
                reserved, reason = None, e.reason
            assert reserved == step["reserved"]
            assert reason == (REFUSALS[step["error"]] if step["error"] else None)
            mapping.finish(op, step["accepted"])
            physical = []
            for p in step["probe"]:
                try:
                    physical.append(mapping.physical([p])[0])
                except ValidationError:
                    physical.append(None)
            assert physical == step["physical"]
            assert mapping.generations.tolist() == step["generations"]
            assert mapping.logical.tolist() == step["logical_map"]


def test_slot_map_refuses_like_the_reference():
    m = SlotMap(8, context=32, offset=3, max_mutations=4)
    with pytest.raises(ValidationError):
        m.reset("A" * 32, 0)  # not a lowercase hex identity
    m.reset("f" * 32, 2)
    with pytest.raises(ValidationError):
        m.reset("f" * 32, 2)  # epochs must grow
    op = Operation("f" * 32, 2, 0, 8)
    with pytest.raises(ValidationError):
        m.prepare([0], [0])  # no active window
    m.begin(op)
    with pytest.raises(ValidationError):
        m.begin(op)  # already active
    with pytest.raises(ValidationError):
        m.reserve([0, 8], [0, 1])  # the same physical slot twice
    with pytest.raises(ValidationError):
        m.reserve([0], [9])  # producing token outside the window
    with pytest.raises(ValidationError):
        m.reserve([0, 1, 2, 3, 4], [0, 1, 2, 3, 4])  # undo capacity
    assert m.reserve([0, 1], [0, 1]) == ([3, 4], [0, 0])
    with pytest.raises(ValidationError):
        m.reserve([2], [0])  # producing tokens do not go backwards
    m.finish(op, 1)
    assert m.physical([0, -1]) == [3, -1]
    with pytest.raises(ValidationError):
        m.physical([1])  # rolled back
    with pytest.raises(ValidationError):
        SlotMap(8, context=4, offset=0)  # context below slots


def test_retained_prefix_keeps_only_validated_rows():
    m = SlotMap(8, context=32, offset=2)
    m.reset("e" * 32, 0)
    op = Operation("e" * 32, 0, 0, 6)
    m.begin(op)
    m.reserve(list(range(6)), list(range(6)))
    m.finish(op, 6)
    m.retain_prefix("e" * 32, 1, 4)
    assert m.physical([0, 1, 2, 3]) == [2, 3, 4, 5]
    assert np.count_nonzero(m.generations) == 4
    with pytest.raises(ValidationError):
        m.physical([4])


WINDOWS = Path(__file__).resolve().parent / "golden" / "slotmap_windows.json"
# each reference refusal message (prefix) and the reasons this module may tag it with
REFUSAL_KINDS = {
    "cache undo row capacity exhausted": {"journal"},
    "one scatter batch repeats a physical cache slot": {"repeat"},
    "cache window is active, stale or exceeds its admitted bounds": {"busy", "stale", "bounds"},
    "cache producing token must be an integer in": {"order", "range"},
}


def _kinds(message):
    return next(kinds for prefix, kinds in REFUSAL_KINDS.items() if message.startswith(prefix))


def test_slot_map_replays_reference_windows():
    """Several batches per window, ring wrap-around with hash-like offsets, refused
    windows and batches, partial acceptance: same slots, refusals, rollback order,
    live rows and per-slot state as the reference's SlotMap at every step."""
    for case in json.loads(WINDOWS.read_text()):
        m = SlotMap(case["slots"], context=case["context"], offset=case["offset"], max_mutations=case["journal"])
        m.reset("e" * 32, 3)
        for step in case["steps"]:
            if step["rows"] > 64 or step["start"] + step["rows"] > case["context"]:
                assert step["begin_error"] is not None
                continue  # Operation() itself refuses rows past the capacity; begin() refuses > 64 rows
            op = Operation("e" * 32, 3, step["start"], step["rows"])
            try:
                m.begin(op)
                began = None
            except ValidationError as e:
                began = e.reason
            if step["begin_error"] is not None:
                assert began in _kinds(step["begin_error"])
                continue
            assert began is None
            for batch in step["batches"]:
                try:
                    got = m.reserve(batch["logical"], batch["tokens"])
                    reserved, reason = [list(map(int, got[0])), list(map(int, got[1]))], None
                except ValidationError as e:
                    reserved, reason = None, e.reason
                assert reserved == batch["reserved"]
                if batch["error"] is None:
                    assert reason is None
                else:
                    assert reason in _kinds(batch["error"]), (reason, batch["error"])
            rejected = [(i, mut.slot, mut.previous_generation) for i, mut in m.rejected(op, step["accepted"])]
            assert rejected == [tuple(r) for r in step["rejected"]]
            m.finish(op, step["accepted"])
            physical = []
            for q in step["probe"]:
                try:
                    physical.append(m.physical([q])[0])
                except ValidationError:
                    physical.append(None)
            assert physical == step["physical"]
            assert m.generations.tolist() == step["generations"]
            assert m.logical.tolist() == step["logical_map"]
