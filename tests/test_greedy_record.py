"""GreedyRunRecord's committed wire format (record_to_json,
src/greedy_run.rs:255-350) against the reference's own committed record
(testdata/gi2-4-greedy-record/record.json, copied unchanged into
tests/golden by make_fixtures.py): the 256-token record parses, its
self-consistency holds as src/greedy_run_test.rs:209-330 checks it, and
re-serializing it gives the file byte for byte. Synthetic records round
trip like src/greedy_run_test.rs:156-207. No GPU.
"""

import hashlib
import json
from pathlib import Path

import pytest

from faber_runtime_b200 import OracleError
from faber_runtime_b200.decoder import (GreedyDivergence, GreedyRunRecord, RECORD_SCHEMA, record_from_json,
                                        record_to_json)

GOLDEN = Path(__file__).resolve().parent / "golden"


def committed():
    raw = (GOLDEN / "greedy_record.json").read_bytes()
    man = json.loads((GOLDEN / "greedy_record_manifest.json").read_text())
    return raw, man


def test_committed_record_is_the_manifest_file_and_self_consistent():
    raw, man = committed()
    assert hashlib.sha256(raw).hexdigest() == man["fixtures"][0]["sha256"]
    record, prompt, trace = record_from_json(raw.decode())
    assert len(record.generated_tokens) == man["fixtures"][0]["generated_token_count"] == 256
    assert record.all_finite and record.first_divergence is None
    assert record.divergence_field() == "none"
    assert trace["file_sha256"] == man["trace"]["file_sha256"]
    assert record.generated_tokens[0] == 30  # top-1 at the prompt end, as the logits golden says


def test_committed_record_reserializes_byte_for_byte():
    raw, _ = committed()
    record, prompt, trace = record_from_json(raw.decode())
    assert record_to_json(record, prompt, trace).encode() == raw


def test_synthetic_record_round_trips_with_its_divergence():
    toks = [30, 198, 198, 504, 808, 6330, 314, 253]
    rec = GreedyRunRecord(toks, True, GreedyDivergence(3, 504, 9, ["top-1", "band"], 0.021))
    wire = record_to_json(rec, [1, 2, 3])
    root = json.loads(wire)
    assert wire.endswith("}\n") and root["schema"] == RECORD_SCHEMA
    assert root["generated_token_count"] == 8 and root["all_finite"] and not root["all_agree"]
    div = root["first_divergence"]
    assert (div["position"], div["comparator_trace_token"], div["oracle_token"]) == (3, 504, 9)
    assert div["failing_thresholds"] == ["top-1", "band"]
    assert rec.divergence_field().startswith("position 3")
    back, prompt, trace = record_from_json(wire)
    assert back == rec and prompt == [1, 2, 3] and trace is None
    ok = GreedyRunRecord(toks[:4], True, None)
    assert json.loads(record_to_json(ok, []))["first_divergence"] is None and ok.divergence_field() == "none"


@pytest.mark.parametrize("edit,kind", [
    (lambda r: r.__setitem__("schema", "other"), "RecordSchema"),
    (lambda r: r["generated_tokens"].__setitem__(5, 7), "RecordHash"),
    (lambda r: r.__setitem__("generated_token_count", 255), "RecordCount"),
    (lambda r: r.__setitem__("all_agree", False), "RecordAgreement"),
])
def test_contradicting_records_are_refused(edit, kind):
    raw, _ = committed()
    root = json.loads(raw)
    edit(root)
    with pytest.raises(OracleError) as e:
        record_from_json(json.dumps(root))
    assert e.value.kind == kind
