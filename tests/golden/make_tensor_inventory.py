"""Writes tests/golden/qwen25_tensors.json: the tensor inventory of the real
Qwen2.5-0.5B checkpoint (name, dtype, shape, and the checkpoint's byte size),
taken from the reference's golden/tensor_digest.json (an independent NumPy
parse of model.safetensors, abho7/llm-inference-webgpu oracle/tensor_digest.py).
The per-tensor SHA-256 digests are left out: they need the weights, which are
not available here.

    python tests/golden/make_tensor_inventory.py /path/to/reference
"""
import json
import os
import sys

ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("B2A_REFERENCE", "")
digest = json.load(open(os.path.join(ref, "golden", "tensor_digest.json")))
out = {
    "source": "golden/tensor_digest.json of the reference (NumPy parse of Qwen2.5-0.5B model.safetensors)",
    "file_bytes": digest["file_bytes"],
    "tensor_count": digest["tensor_count"],
    "tensors": {name: {"dtype": t["dtype"], "shape": t["shape"]} for name, t in sorted(digest["tensors"].items())},
}
path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "qwen25_tensors.json")
with open(path, "w") as f:
    json.dump(out, f, indent=0, sort_keys=True)
print(path, out["tensor_count"])
