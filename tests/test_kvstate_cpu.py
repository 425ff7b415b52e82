"""Host logic of the KV state boundary: snapshot record checks (the
reference's alpaccaroo/memory.py:634-690 rules for attention layers) and
the record format pinned by the reference's own snapshot
(tests/golden/kv_state.npz, written by alpaccaroo.memory.FullAttentionState)."""
import numpy as np
import pytest

from alpacca_open_sourced_by_jt_b200.kvstate import (AttentionSnapshot, SnapshotMismatchError,
                                                     StateError, validate_snapshot)
from tests.golden import cases


def _snap(L=3, KV=2, D=4, **kw):
    base = dict(layer_index=1, logical_length=L, kv_heads=KV, key_dim=D, value_dim=D,
                key=bytes(L * KV * D * 4), value=bytes(L * KV * D * 4))
    base.update(kw)
    return AttentionSnapshot(**base)


def _check(s, capacity=8):
    validate_snapshot(s, layer_index=1, kv_heads=2, key_dim=4, value_dim=4, capacity=capacity)


def test_valid_record_passes():
    _check(_snap())
    _check(_snap(L=0, key=b"", value=b""))


@pytest.mark.parametrize("change,err", [
    (dict(layer_index=2), SnapshotMismatchError),
    (dict(kind="recurrent"), SnapshotMismatchError),
    (dict(dtype="f16-le"), SnapshotMismatchError),
    (dict(kv_heads=3), SnapshotMismatchError),
    (dict(value_dim=5), SnapshotMismatchError),
    (dict(key=bytes(10)), StateError),
    (dict(value=bytes(3 * 2 * 4 * 4 + 4)), StateError),
])
def test_bad_records_are_rejected(change, err):
    with pytest.raises(err):
        _check(_snap(**change))


def test_capacity_is_enforced():
    with pytest.raises(SnapshotMismatchError):
        _check(_snap(L=9, key=bytes(9 * 32), value=bytes(9 * 32)), capacity=8)


def test_record_format_matches_reference_golden(golden):
    g = golden("kv_state.npz")
    c = cases.kv_state_case()
    assert c["sha256"] == str(g["input_sha256"])
    assert str(g["dtype"]) == "f32-le" and str(g["kind"]) == "attention"
    # the reference's payload is the rows' float32 little-endian bytes
    assert g["key"].tobytes() == c["k"].astype("<f4").tobytes()
    assert g["value"].tobytes() == c["v"].astype("<f4").tobytes()
    n = c["truncate"]
    assert g["key_cut"].tobytes() == c["k"][:n].astype("<f4").tobytes()
    assert int(g["memory_bytes"]) == 2 * c["k"].size * 4
    s = AttentionSnapshot(layer_index=c["layer_index"], logical_length=c["L"],
                          kv_heads=c["KV"], key_dim=c["D"], value_dim=c["D"],
                          key=g["key"].tobytes(), value=g["value"].tobytes())
    assert s.memory_bytes() == int(g["memory_bytes"])
    validate_snapshot(s, layer_index=c["layer_index"], kv_heads=c["KV"], key_dim=c["D"],
                      value_dim=c["D"], capacity=c["L"])
