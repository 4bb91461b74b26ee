"""Writes tests/golden/laguna_inventory_golden.json from the reference's
public tensor-inventory fixture (fixtures/poolside_laguna_xs_2_1_nvfp4_tensor_
inventory.json): digests and counts only, no tensor list, so that the loader's
restatement of the inventory (checkpoint.expected_inventory) and its
canonical hash are pinned without the reference tree.

  python tests/golden/make_inventory_golden.py /path/to/reference
"""
import hashlib
import json
import os
import sys

ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
inv = json.load(open(os.path.join(
    ref, "fixtures", "poolside_laguna_xs_2_1_nvfp4_tensor_inventory.json")))
rows = sorted(inv["tensors"], key=lambda r: r[0])  # [name, dtype, shape, shard index]
h = hashlib.sha256()
for name, dtype, shape, _ in rows:
    h.update(json.dumps([name, dtype, shape], separators=(",", ":")).encode() + b"\n")
out = {
    "source": "fixtures/poolside_laguna_xs_2_1_nvfp4_tensor_inventory.json (summary)",
    "tensor_count": inv["summary"]["tensor_count"],
    "dtype_counts": inv["summary"]["dtype_counts"],
    "canonical_sha256_with_shards": inv["summary"]["canonical_sha256"],
    "sha256_name_dtype_shape": h.hexdigest(),
}
path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "laguna_inventory_golden.json")
json.dump(out, open(path, "w"), indent=1)
print(path, out)
