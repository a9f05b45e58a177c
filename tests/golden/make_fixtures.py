"""Regenerate the committed golden fixtures from faber-runtime's testdata.

Reads the reference's self-contained per-op goldens
(testdata/gi2-2-op-goldens/*.json: input f32 bits, expected output f32 bits,
SHA-256 in manifest.json) and the prompt-end logits golden
(testdata/gi2-3-logits-golden/logits-pos0.json), verifies every SHA-256 the
reference manifest records, and writes:

  op_goldens.npz   - float32 arrays "<op>.<input name>" and "<op>.expected"
  op_goldens.json  - per-op scalar parameters, input names, expected SHA-256
  logits_pos0.npz  - "raw_logits" (49152 f32), "logp", top-1 ids
  greedy_record.json           - the committed 256-token greedy run record
                                 (testdata/gi2-4-greedy-record/record.json, bytes unchanged)
  greedy_record_manifest.json  - its manifest (SHA-256, token count)

Run from the repository root in an environment that has the reference tree,
giving the path of the faber-runtime checkout as the first argument:
    python tests/golden/make_fixtures.py <faber-runtime checkout>
    python tests/golden/make_fixtures.py <faber-runtime checkout> record   # the record files only
The GPU-side tests read only the outputs, never the reference tree.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OPS = ["rms_norm", "dense", "rope", "attention", "residual", "swiglu"]


def _f32(hexstr: str) -> np.ndarray:
    return np.frombuffer(bytes.fromhex(hexstr), dtype="<f4").astype(np.float32)


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    gdir = ref / "testdata" / "gi2-2-op-goldens"
    manifest = json.loads((gdir / "manifest.json").read_text())
    file_sha = {f["op"]: f["sha256"] for f in manifest["fixtures"]}
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    for op in OPS:
        raw = (gdir / f"{op}.json").read_bytes()
        assert hashlib.sha256(raw).hexdigest() == file_sha[op], f"{op}.json sha256 mismatch"
        fx = json.loads(raw)
        inputs = []
        for inp in fx["inputs"]:
            a = _f32(inp["f32_le_hex"])
            assert a.size == inp["elements"]
            arrays[f"{op}.{inp['name']}"] = a
            inputs.append(inp["name"])
        exp = fx["expected_output"]
        e = _f32(exp["f32_le_hex"])
        assert e.size == exp["elements"]
        assert hashlib.sha256(e.astype("<f4").tobytes()).hexdigest() == exp["sha256"]
        arrays[f"{op}.expected"] = e
        params = {k: v for k, v in fx.items()
                  if k not in ("inputs", "expected_output", "model", "pinned_position",
                               "coverage_ok", "generator", "schema")}
        meta[op] = {"inputs": inputs, "expected_name": exp["name"],
                    "expected_sha256": exp["sha256"], "file_sha256": file_sha[op],
                    "params": params}
    np.savez_compressed(HERE / "op_goldens.npz", **arrays)
    (HERE / "op_goldens.json").write_text(json.dumps(
        {"source": "faber-runtime testdata/gi2-2-op-goldens",
         "generator": manifest["generator"], "pinned_position": manifest["pinned_position"],
         "ops": meta}, indent=1, sort_keys=True) + "\n")

    ldir = ref / "testdata" / "gi2-3-logits-golden"
    lman = json.loads((ldir / "manifest.json").read_text())
    raw = (ldir / "logits-pos0.json").read_bytes()
    assert hashlib.sha256(raw).hexdigest() == lman["fixtures"][0]["sha256"]
    lg = json.loads(raw)
    np.savez_compressed(
        HERE / "logits_pos0.npz",
        raw_logits=_f32(lg["raw_logits"]["f32_le_hex"]),
        logp=_f32(lg["logp"]["f32_le_hex"]),
        raw_argmax=np.int64(int(lg["raw_argmax"])),
        top1_non_eog=np.int64(int(lg["top1_non_eog"])),
    )
    print("wrote", HERE / "op_goldens.npz", HERE / "logits_pos0.npz")


def record(ref_root: str) -> None:
    rdir = Path(ref_root) / "testdata" / "gi2-4-greedy-record"
    man = json.loads((rdir / "manifest.json").read_text())
    raw = (rdir / "record.json").read_bytes()
    assert hashlib.sha256(raw).hexdigest() == man["fixtures"][0]["sha256"], "record.json sha256 mismatch"
    (HERE / "greedy_record.json").write_bytes(raw)
    (HERE / "greedy_record_manifest.json").write_text(json.dumps(man, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "greedy_record.json")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_fixtures.py <faber-runtime checkout> [record]")
    root = sys.argv[1]
    if len(sys.argv) > 2 and sys.argv[2] == "record":
        record(root)
    else:
        main(root)
        record(root)
