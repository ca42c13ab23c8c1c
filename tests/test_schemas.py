"""The op schemas this package defines are the reference's: every entry of
voyager_b200.ops.SCHEMAS, parsed by torch, equals the schema torch parsed
from the reference's own torch.library definitions (recorded by
tests/golden/make_golden.py in schemas.json), so exported graphs dispatch
here unchanged."""

import json
import os

import torch

from voyager_b200 import ops

HERE = os.path.dirname(os.path.abspath(__file__))


def test_schemas_equal_the_reference():
    ref = json.load(open(os.path.join(HERE, "golden", "schemas.json")))
    assert len(ops.SCHEMAS) >= 13
    for name, schema in ops.SCHEMAS.items():
        assert name in ref, f"{name} is not an op of the reference"
        ours = str(torch._C.parse_schema("quantized_ops::" + schema))
        assert ours == ref[name], (name, ours, ref[name])


def test_registered_ops_use_those_schemas():
    # the live op objects in this process carry the same schemas
    ref = json.load(open(os.path.join(HERE, "golden", "schemas.json")))
    import voyager_b200  # noqa: F401

    for name in ops.SCHEMAS:
        assert str(getattr(torch.ops.quantized_ops, name).default._schema) == ref[name]
