"""The C++ loader and operator registry (no GPU): mirrors the reference's
import smoke test (tests/onnx/test_onnx_import.cpp:141-197) — parse a model,
check registration and node counts — through the lcml_session C ABI."""
import base64
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def _net(text):
    from luisaml_b200.session import Network
    return Network(text)


def test_reference_fixture_loads():
    text = open(os.path.join(GOLDEN, "simple_mlp", "simple_mlp.onnx.json")).read()
    net = _net(text)
    assert net.info() == (5, 1, 1)  # Gemm, Relu, Gemm, Relu, Gemm


def test_inline_model_and_registry():
    from luisaml_b200 import session
    assert session.load().lcml_opset_size() >= 20
    zeros = base64.b64encode(np.zeros(4 * 3, dtype=np.float32).tobytes()).decode()
    g = {"name": "tiny", "input": [{"name": "x", "type": {"tensor_type": {"elem_type": "FLOAT", "shape": {"dim": [{"dim_value": "1"}, {"dim_value": "4"}]}}}}],
         "output": [{"name": "y", "type": {"tensor_type": {"elem_type": "FLOAT", "shape": {"dim": [{"dim_value": "1"}, {"dim_value": "3"}]}}}}],
         "initializer": [{"name": "w", "data_type": "FLOAT", "dims": ["3", "4"], "raw_data": zeros}],
         "value_info": [{"name": "h", "type": {"tensor_type": {"elem_type": "FLOAT", "shape": {"dim": [{"dim_value": "1"}, {"dim_value": "3"}]}}}}],
         "node": [{"input": ["x", "w"], "output": ["h"], "name": "g", "op_type": "Gemm",
                   "attribute": [{"name": "transB", "i": "1", "type": "INT"}]},
                  {"input": ["h"], "output": ["y"], "name": "r", "op_type": "Relu"}]}
    net = _net(json.dumps({"ir_version": "10", "producer_name": "t", "producer_version": "0", "graph": g}))
    assert net.info() == (2, 1, 1)
    g["node"][1]["op_type"] = "NotAnOp"
    with pytest.raises(Exception, match="Operator not found: NotAnOp"):
        _net(json.dumps({"ir_version": "10", "producer_name": "t", "producer_version": "0", "graph": g}))


def test_qdq_mlp_graph_loads():
    from luisaml_b200 import graphs
    text, blob, meta = graphs.mlp()
    net = _net(text)
    assert net.info() == (8, 1, 1)  # 3 DequantizeLinear + 3 Gemm + 2 Relu
    assert len(blob) % 4 == 0 and len(meta["layers"]) == 3


def test_host_encoder_matches_golden():
    from luisaml_b200 import export
    for name in ("e4m3_encode_structured.npz", "e4m3_encode_random.npz"):
        d = np.load(os.path.join(GOLDEN, name))
        assert np.array_equal(export.e4m3_encode(d["x"]), d["q"])
