"""Extract the reference's own golden values for the verify path into reference_goldens.json.

Reads mlx-dspark's tests/test_batch_engine.py as text (``ast``; nothing of the reference is
imported or executed — it needs MLX, which is not available here) and records, per test, the
operation sequence the test performs and the expected integer values it asserts. The
operation sequences are transcribed below; every expected value is taken from the test
source's own literals, in the order they appear, so a change in the reference's goldens
changes the fixture.

Usage: python tests/golden/extract_reference_goldens.py path/to/mlx-dspark/tests
"""

from __future__ import annotations

import ast
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
STEP = 256  # src/mlx_dspark/batch_engine.py:38


def _literals(fn: ast.FunctionDef) -> list:
    """Integer-list literals of every ``assert`` in the function, in source order."""
    out = []
    for node in ast.walk(fn):
        if isinstance(node, ast.Assert):
            for sub in ast.walk(node.test):
                if isinstance(sub, (ast.List, ast.Tuple)):
                    try:
                        val = ast.literal_eval(sub)
                    except ValueError:
                        continue
                    if all(isinstance(v, int) for v in val) or all(
                            isinstance(v, list) for v in val):
                        out.append(list(val) if isinstance(val, tuple) else val)
    out.sort(key=lambda v: 0)  # stable: ast.walk order within an assert is source order
    return out


def _asserts_in_order(fn: ast.FunctionDef) -> list:
    vals = []
    for stmt in fn.body:
        for node in ast.walk(stmt):
            if isinstance(node, ast.Assert):
                for sub in ast.walk(node.test):
                    if isinstance(sub, (ast.List, ast.Tuple)):
                        try:
                            v = ast.literal_eval(sub)
                        except ValueError:
                            continue
                        vals.append(list(v))
    return vals


def main(ref_tests: Path) -> dict:
    src = (ref_tests / "test_batch_engine.py").read_text()
    tree = ast.parse(src)
    fns = {n.name: n for n in tree.body if isinstance(n, ast.FunctionDef)}

    def lits(name):
        return _asserts_in_order(fns[name])

    cases = []
    v = lits("test_offset_property_matches_offsets")
    cases.append({"name": "offset_property", "lens": [3, 1, 4], "ops": [["expect", v[0]]]})
    v = lits("test_update_and_fetch_writes_at_each_row_offset")
    cases.append({"name": "update_at_row_offsets", "lens": [3, 1, 4],
                  "ops": [["update", 1, 5], ["expect", v[0]]]})
    v = lits("test_multi_token_update")
    cases.append({"name": "multi_token_update", "lens": [2, 2, 2],
                  "ops": [["update", 3], ["expect", v[0]]]})
    v = lits("test_trim_is_per_row_metadata_and_next_write_overwrites")
    cases.append({"name": "trim_then_overwrite", "lens": [4, 4, 4],
                  "ops": [["update", 1], ["expect", v[0]], ["trim", [0, 1, 2]],
                          ["expect", v[1]], ["update", 1], ["expect", v[2]]]})
    v = lits("test_trim_clamps_at_zero")
    cases.append({"name": "trim_clamps", "lens": [2, 1, 3],
                  "ops": [["trim", [5, 0, 1]], ["expect", v[0]]]})
    v = lits("test_move_row_compacts_and_vacates")
    cases.append({"name": "move_row", "lens": [3, 2, 4], "ops": [["move", 2, 0], ["expect", v[0]]]})
    v = lits("test_rows_view_narrows_offset_and_update")
    cases.append({"name": "rows_view", "lens": [3, 1, 4],
                  "ops": [["rows", 2], ["update", 1, 4], ["expect", v[1]]],
                  "offset_view": v[0]})
    cases.append({"name": "grows_buffer", "lens": [STEP - 1, STEP - 1],
                  "ops": [["update", 3], ["expect", [STEP + 2, STEP + 2]]]})

    masks = []
    v = lits("test_build_batch_mask_causal_and_padding")
    masks.append({"offsets": [2, 0], "T": 2, "shape": v[0],
                  "index": [[0, 0], [0, 1], [1, 0], [1, 1]], "rows": v[1:5]})
    v = lits("test_build_batch_mask_single_token_decode")
    masks.append({"offsets": [5, 3, 0], "T": 1, "shape": v[0],
                  "index": [[0, 0], [1, 0], [2, 0]], "rows": v[1:4]})
    v = lits("test_ctx_block_mask_hides_context_padding")
    ctx = [{"lens": [2, 0], "k": 2, "shape": v[0], "index": [[0, 0], [1, 0]], "rows": v[1:3]}]
    v = lits("test_batched_sample_block_no_markov_is_argmax")
    sample = [{"hot": [[0, 0, 2], [0, 1, 4], [0, 2, 1], [1, 0, 0], [1, 1, 3], [1, 2, 2]],
               "shape": [2, 3, 5], "argmax": v[0]}]
    return {"source": "mlx-dspark tests/test_batch_engine.py", "step": STEP,
            "batch_cache": cases, "batch_mask": masks, "ctx_block_mask": ctx,
            "sample_block_argmax": sample}


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: extract_reference_goldens.py path/to/mlx-dspark/tests")
    ref = Path(sys.argv[1])
    data = main(ref)
    (HERE / "reference_goldens.json").write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {HERE / 'reference_goldens.json'}")
