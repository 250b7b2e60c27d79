import json

import pytest

from vericcl_b200.errors import InputValidationError
from vericcl_b200.examples import example_documents, write_documents
from vericcl_b200.input.loader import load_request, parse_override, resolve_documents
from vericcl_b200.input.schema import SCHEMAS, json_schema


def docs(**kw):
    return example_documents("allreduce", "hierarchy", 4, **kw)


def test_resolves_and_records_sources():
    req = resolve_documents(docs())
    assert req.rank_count == 4
    assert req.hyperparameters.slice_count == 4
    assert req.value_sources["sketch.collective.datatype"]["kind"] == "input"
    assert req.value_sources["runtime.tb_layout"]["kind"] == "default"
    assert req.size_accounting["valid_output_bytes"] == 1 << 20


def test_rejects_unknown_field():
    d = docs()
    d["sketch"]["collective"]["bogus"] = 1
    with pytest.raises(InputValidationError, match="unknown fields"):
        resolve_documents(d)


def test_rejects_duplicate_keys(tmp_path):
    files = write_documents(tmp_path, docs())
    text = files["atom"].read_text()
    files["atom"].write_text(text.replace('"synthesis_method"', '"M_switch": 5, "synthesis_method"', 1)
                             .replace('"M_switch": 16777216', '"M_switch": 16777216, "M_switch": 3', 1))
    with pytest.raises(InputValidationError, match="duplicate"):
        load_request(files)


def test_rejects_non_finite(tmp_path):
    files = write_documents(tmp_path, docs())
    data = files["topology"].read_text().replace('"alpha_us": 1.5', '"alpha_us": NaN', 1)
    files["topology"].write_text(data)
    with pytest.raises(InputValidationError, match="non-finite"):
        load_request(files)


def test_slice_must_divide_size():
    d = docs(total_size_bytes=1000, slice_size_bytes=300)
    with pytest.raises(InputValidationError, match="divide"):
        resolve_documents(d)


def test_override_fills_but_does_not_replace_without_flag():
    d = docs()
    req = resolve_documents(d, overrides=["sketch.trace_and_measure.pairs=4"])
    assert req.request_config["sketch"]["trace_and_measure"]["pairs"] == 4
    with pytest.raises(InputValidationError, match="override-input"):
        resolve_documents(d, overrides=["sketch.collective.datatype=\"bfloat16\""])
    req = resolve_documents(d, overrides=["sketch.collective.datatype=\"bfloat16\""], override_input=True)
    assert req.collective.datatype == "bfloat16"
    assert req.value_sources["sketch.collective.datatype"]["kind"] == "override"


def test_auto_method_uses_m_switch():
    d = docs()
    d["atom"]["synthesis_method"] = "auto"
    d["atom"]["M_switch"] = 1 << 10
    assert resolve_documents(d).selected_synthesis_method == "constructive_trees"
    d["atom"]["M_switch"] = 1 << 30
    assert resolve_documents(d).selected_synthesis_method == "hierarchy"


def test_operator_alias_and_root_rules():
    d = docs()
    d["sketch"]["collective"]["operator"] = "ALL_REDUCE"
    assert resolve_documents(d).collective.kind.value == "allreduce"
    d = example_documents("allgather", "hierarchy", 4)
    d["sketch"]["collective"]["reduction_op"] = "sum"
    with pytest.raises(InputValidationError, match="not applicable"):
        resolve_documents(d)


def test_rank_map_must_cover_ranks():
    d = docs()
    d["runtime"]["rank_map"] = d["runtime"]["rank_map"][:3]
    with pytest.raises(InputValidationError, match="rank_map"):
        resolve_documents(d)


def test_forbidden_transfer_expansion():
    d = docs()
    d["atom"]["forbidden_transfers"] = [[0, 1, 2, 0]]
    req = resolve_documents(d)
    assert len(req.atom_constraints.forbidden_transfers) == 1
    assert req.hyperparameters.reference_slice_size_bytes == req.hyperparameters.slice_size_bytes


def test_parse_override():
    path, value = parse_override("sketch.budgets.max_tuning_rounds=3")
    assert path == ("sketch", "budgets", "max_tuning_rounds") and value == 3
    with pytest.raises(InputValidationError):
        parse_override("nope")


def test_json_schema_export():
    for name, node in SCHEMAS.items():
        schema = json_schema(node, name)
        assert schema["type"] == "object"
        json.dumps(schema)


def test_committed_schema_files_and_docs_are_current():
    """schemas/*.schema.json and docs/input-schema.md match what the schema DSL generates."""
    from vericcl_b200.input.docs import stale
    assert stale() == []
