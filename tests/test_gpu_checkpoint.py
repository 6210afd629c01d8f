"""A pre-quantized int8 checkpoint (tendo_b200/checkpoint.py) round trip on
the GPU: the synthetic tiny model exported to safetensors and loaded into a
fresh engine decodes the golden greedy tokens (the oracle's)."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_export_load_greedy(tb, cuda, tmp_path):
    from tendo_b200 import checkpoint as ck

    with open(os.path.join(HERE, "golden", "tiny_greedy.json")) as f:
        golden = json.load(f)
    src = tb.QuantizedModel(golden["config"], batch=1, device=0)
    src.init_synthetic(golden["weight_seed"])
    path = str(tmp_path / "tiny.safetensors")
    ck.export_model(src, path)
    src.close()
    dst = tb.QuantizedModel(golden["config"], batch=1, device=0)
    ck.load_model(dst, path)
    toks = dst.generate_greedy(np.array(golden["prompt"]), 32)
    np.testing.assert_array_equal(toks[0], np.array(golden["tokens"][:32]))
    dst.close()
