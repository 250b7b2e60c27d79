"""Generate the public input contract files from the schema DSL.

    python -m vericcl_b200.input.docs [--check]

Writes ``schemas/<document>.schema.json`` (JSON Schema 2020-12) and
``docs/input-schema.md`` (one table per document: field path, type, default,
purpose) from :mod:`vericcl_b200.input.schema`; ``--check`` only reports
whether the committed files are current (exit 1 when stale).  Reference
counterpart: tools/generate_schema_docs.py.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

from vericcl_b200.input import schema as S

ROOT = Path(__file__).resolve().parents[2]
DOCUMENTS = (("topology", S.TOPOLOGY), ("sketch", S.SKETCH), ("atom", S.ATOM), ("runtime", S.RUNTIME))


def _default(node) -> str:
    if node.default is S._ABSENT:
        return ""
    return json.dumps(node.default)


def render_markdown() -> str:
    lines = ["# Input field reference", "",
             "Generated from `vericcl_b200/input/schema.py` (`json_schema`, `field_rows`).", ""]
    for name, node in DOCUMENTS:
        lines += ["## %s.json" % name, "", "| Field | Type | Default | Purpose |", "|---|---|---|---|"]
        for path, child in S.field_rows(node, name):
            if path == name:
                continue
            lines.append("| `%s` | %s | %s | %s |" % (path, child.kind, _default(child), child.doc))
        lines.append("")
    return "\n".join(lines)


def render_schemas() -> dict:
    return {name: json.dumps(S.json_schema(node, name), indent=2, sort_keys=True) + "\n" for name, node in DOCUMENTS}


def outputs(root: Path = ROOT) -> dict:
    files = {root / "docs" / "input-schema.md": render_markdown()}
    for name, text in render_schemas().items():
        files[root / "schemas" / ("%s.schema.json" % name)] = text
    return files


def stale(root: Path = ROOT) -> list:
    return [str(p.relative_to(root)) for p, text in outputs(root).items()
            if not p.exists() or p.read_text() != text]


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if "-h" in argv or "--help" in argv:
        print("usage: python -m vericcl_b200.input.docs [--check]\n"
              "regenerates docs/input-schema.md and schemas/*.schema.json from the input schema; --check only "
              "lists the files that are out of date (exit 1 when any is)")
        return 0
    if "--check" in argv:
        bad = stale()
        for path in bad:
            print("stale: %s" % path)
        return 1 if bad else 0
    for path, text in outputs().items():
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(text)
        print("wrote %s" % path.relative_to(ROOT))
    return 0


if __name__ == "__main__":
    sys.exit(main())
