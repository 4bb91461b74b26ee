"""Laguna XS 2.1 NVFP4 checkpoint reader: safetensors shards + index, the
weight contract's validation, and the sparse layers' tensors in the layout the
kernels read (the stored layout, unchanged).

Contract (the reference's docs/laguna-weight-contract.md):
* directory: config.json, model.safetensors.index.json, the shards it names
  (:35-55): every referenced shard exists, every present shard is referenced,
  each shard holds exactly the tensors the index assigns it, names are unique,
  rotary_emb.inv_freq tables are excluded;
* config: `quantization` and `quantization_config` both present, equal, and
  exactly {"group_size": 16, "bits": 4, "mode": "nvfp4"} (:57-66);
* only routed and shared expert projections are quantized: `<stem>.weight`
  U32 [..., rows, in / 8] and `<stem>.scales` U8 [..., rows, in / 16], no
  `.biases` (:68-78);
* the tensor inventory (:80-127), which `expected_inventory` restates from
  the config's geometry.

The safetensors container: an 8-byte little-endian header length N, N bytes
of JSON ({name: {"dtype", "shape", "data_offsets": [begin, end]}} plus an
optional "__metadata__"), then the data; offsets are relative to the first
data byte.  Tensors are read through a memory map, so loading one layer
touches only that layer's bytes.

`interleave_gate_up` / `split_gate_up` are the reference runtime's offline
[gate32, up32] row-tile interleave of the routed gate/up banks
(Sources/MLXFastModel/LagunaRuntimeModel.swift:10605-10625) and its inverse:
the kernels here read gate and up as separate banks, so a fused bank is split
on load.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass

import numpy as np
import torch

from .laguna import LagunaMoEConfig

NVFP4_QUANT = {"group_size": 16, "bits": 4, "mode": "nvfp4"}

# safetensors dtype name -> (numpy dtype, torch dtype)
_DTYPES = {
    "BF16": (np.uint16, torch.bfloat16),
    "F16": (np.float16, torch.float16),
    "F32": (np.float32, torch.float32),
    "F64": (np.float64, torch.float64),
    "U8": (np.uint8, torch.uint8),
    "I8": (np.int8, torch.int8),
    "U16": (np.uint16, torch.uint16),
    "I16": (np.int16, torch.int16),
    "U32": (np.uint32, torch.uint32),
    "I32": (np.int32, torch.int32),
    "U64": (np.uint64, torch.uint64),
    "I64": (np.int64, torch.int64),
}
_TORCH_TO_ST = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32",
                torch.float64: "F64", torch.uint8: "U8", torch.int8: "I8",
                torch.uint16: "U16", torch.int16: "I16", torch.uint32: "U32",
                torch.int32: "I32", torch.uint64: "U64", torch.int64: "I64"}


class CheckpointError(ValueError):
    """The directory does not satisfy the weight contract."""


# --------------------------------------------------------------------------
# safetensors container
# --------------------------------------------------------------------------

class SafetensorsFile:
    """One shard: its header, and tensors read through a memory map."""

    def __init__(self, path: str):
        self.path = path
        size = os.path.getsize(path)
        with open(path, "rb") as f:
            head = f.read(8)
            if len(head) != 8:
                raise CheckpointError(f"{path}: shorter than a safetensors header")
            (n,) = struct.unpack("<Q", head)
            if n > size - 8:
                raise CheckpointError(f"{path}: header length {n} beyond the file")
            try:
                header = json.loads(f.read(n).decode("utf-8"))
            except (UnicodeDecodeError, json.JSONDecodeError) as e:
                raise CheckpointError(f"{path}: header is not JSON ({e})") from None
        self.metadata = header.pop("__metadata__", None) or {}
        self.data_start = 8 + n
        self.tensors = {}
        for name, info in header.items():
            dt = info.get("dtype")
            if dt not in _DTYPES:
                raise CheckpointError(f"{path}: {name}: unknown dtype {dt!r}")
            shape = tuple(int(d) for d in info.get("shape", ()))
            b, e = (int(v) for v in info["data_offsets"])
            count = int(np.prod(shape, dtype=np.int64)) if shape else 1
            if e - b != count * np.dtype(_DTYPES[dt][0]).itemsize or b < 0 or \
                    self.data_start + e > size:
                raise CheckpointError(f"{path}: {name}: data_offsets [{b}, {e}] do not "
                                      f"hold {dt} {list(shape)}")
            self.tensors[name] = (dt, shape, b, e)
        self._map = None

    def names(self):
        return list(self.tensors)

    def info(self, name):
        dt, shape, _, _ = self.tensors[name]
        return dt, shape

    def numpy(self, name) -> np.ndarray:
        """The tensor as a read-only numpy view of the memory map (BF16 as its
        uint16 bits)."""
        if self._map is None:
            self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        dt, shape, b, e = self.tensors[name]
        raw = self._map[self.data_start + b:self.data_start + e]
        return raw.view(_DTYPES[dt][0]).reshape(shape)

    def tensor(self, name, device="cpu") -> torch.Tensor:
        dt = self.tensors[name][0]
        a = np.array(self.numpy(name))  # one copy out of the map (writable)
        t = torch.from_numpy(a)
        if dt == "BF16":
            t = t.view(torch.bfloat16)
        return t.to(device)


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Write `tensors` (name -> CPU-copyable torch tensor) as one safetensors
    file, in name order, each tensor's data 8-byte aligned."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if t.dtype not in _TORCH_TO_ST:
            raise TypeError(f"{name}: dtype {t.dtype} has no safetensors name")
        dt = _TORCH_TO_ST[t.dtype]
        npdt = _DTYPES[dt][0]
        raw = (t.view(torch.uint16) if t.dtype == torch.bfloat16 else t).numpy().astype(
            npdt, copy=False).tobytes()
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        pad = (-len(raw)) % 8
        blobs.append(raw + b"\0" * pad)  # the recorded end stays exact; pad between tensors
        off += len(raw) + pad
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


# --------------------------------------------------------------------------
# the inventory the contract names
# --------------------------------------------------------------------------

@dataclass(frozen=True)
class LagunaGeometry:
    """The whole-model geometry the inventory depends on (config.json keys)."""
    hidden: int
    vocab: int
    num_layers: int
    head_dim: int
    kv_heads: int
    heads_per_layer: tuple
    mlp_layer_types: tuple
    dense_inter: int
    moe: LagunaMoEConfig

    @staticmethod
    def from_config(cfg: dict) -> "LagunaGeometry":
        L = int(cfg["num_hidden_layers"])
        heads = cfg.get("num_attention_heads_per_layer") or [cfg["num_attention_heads"]] * L
        kinds = cfg.get("mlp_layer_types")
        if kinds is None:
            dense = set(cfg.get("mlp_only_layers", []))
            kinds = ["dense" if i in dense else "sparse" for i in range(L)]
        if len(heads) != L or len(kinds) != L:
            raise CheckpointError("per-layer lists do not have num_hidden_layers entries")
        moe = LagunaMoEConfig(
            hidden=int(cfg["hidden_size"]), inter=int(cfg["moe_intermediate_size"]),
            n_experts=int(cfg["num_experts"]), top_k=int(cfg["num_experts_per_tok"]),
            shared_inter=int(cfg.get("shared_expert_intermediate_size", 0)),
            routed_scaling=float(cfg.get("moe_routed_scaling_factor", 1.0)),
            norm_topk_prob=bool(cfg.get("norm_topk_prob", True)), num_layers=L,
            num_sparse_layers=sum(1 for k in kinds if k == "sparse"),
            rms_norm_eps=float(cfg.get("rms_norm_eps", 1e-6)))
        return LagunaGeometry(hidden=moe.hidden, vocab=int(cfg["vocab_size"]), num_layers=L,
                              head_dim=int(cfg["head_dim"]),
                              kv_heads=int(cfg["num_key_value_heads"]),
                              heads_per_layer=tuple(int(h) for h in heads),
                              mlp_layer_types=tuple(kinds),
                              dense_inter=int(cfg["intermediate_size"]), moe=moe)

    def sparse_layers(self):
        return [i for i, k in enumerate(self.mlp_layer_types) if k == "sparse"]


def _quantized(stem, rows_shape, k_in):
    return [(f"{stem}.weight", "U32", (*rows_shape, k_in // 8)),
            (f"{stem}.scales", "U8", (*rows_shape, k_in // 16))]


def expected_inventory(g: LagunaGeometry):
    """Every (name, dtype, shape) the contract requires for geometry g, in
    name order: embeddings, final norm and untied lm_head; per layer the two
    norms and the gated attention projections; the dense MLP in dense layers;
    in sparse layers the router, its correction bias, and the NVFP4 routed and
    shared expert projections."""
    H, D = g.hidden, g.head_dim
    out = [("model.embed_tokens.weight", "BF16", (g.vocab, H)),
           ("model.norm.weight", "BF16", (H,)),
           ("lm_head.weight", "BF16", (g.vocab, H))]
    m = g.moe
    for n in range(g.num_layers):
        p = f"model.layers.{n}"
        q = g.heads_per_layer[n]
        out += [(f"{p}.input_layernorm.weight", "BF16", (H,)),
                (f"{p}.post_attention_layernorm.weight", "BF16", (H,)),
                (f"{p}.self_attn.q_proj.weight", "BF16", (q * D, H)),
                (f"{p}.self_attn.k_proj.weight", "BF16", (g.kv_heads * D, H)),
                (f"{p}.self_attn.v_proj.weight", "BF16", (g.kv_heads * D, H)),
                (f"{p}.self_attn.o_proj.weight", "BF16", (H, q * D)),
                (f"{p}.self_attn.g_proj.weight", "BF16", (q, H)),
                (f"{p}.self_attn.q_norm.weight", "BF16", (D,)),
                (f"{p}.self_attn.k_norm.weight", "BF16", (D,))]
        if g.mlp_layer_types[n] == "dense":
            out += [(f"{p}.mlp.gate_proj.weight", "BF16", (g.dense_inter, H)),
                    (f"{p}.mlp.up_proj.weight", "BF16", (g.dense_inter, H)),
                    (f"{p}.mlp.down_proj.weight", "BF16", (H, g.dense_inter))]
        else:
            E, I, Is = m.n_experts, m.inter, m.shared_inter
            out += [(f"{p}.mlp.gate.weight", "BF16", (E, H)),
                    (f"{p}.mlp.gate.e_score_correction_bias", "F32", (E,))]
            out += _quantized(f"{p}.mlp.switch_mlp.gate_proj", (E, I), H)
            out += _quantized(f"{p}.mlp.switch_mlp.up_proj", (E, I), H)
            out += _quantized(f"{p}.mlp.switch_mlp.down_proj", (E, H), I)
            if Is:
                out += _quantized(f"{p}.mlp.shared_expert.gate_proj", (Is,), H)
                out += _quantized(f"{p}.mlp.shared_expert.up_proj", (Is,), H)
                out += _quantized(f"{p}.mlp.shared_expert.down_proj", (H,), Is)
    return sorted(out)


def canonical_inventory_sha256(entries) -> str:
    """SHA-256 of the inventory in the reference fixture's canonical form:
    entries sorted by name, each encoded as compact JSON
    [name, dtype, shape(, shard)] followed by a line feed."""
    h = hashlib.sha256()
    for e in sorted(entries, key=lambda e: e[0]):
        row = [e[0], e[1], list(e[2])] + list(e[3:])
        h.update(json.dumps(row, separators=(",", ":"), ensure_ascii=False).encode("utf-8"))
        h.update(b"\n")
    return h.hexdigest()


# --------------------------------------------------------------------------
# the [gate32, up32] interleave
# --------------------------------------------------------------------------

def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, pair_rows: int = 32) -> torch.Tensor:
    """Fused routed gate/up bank [E, 2 I, D] from gate and up [E, I, D]
    (packed codes or scale bytes alike): row tile t of pair_rows gate rows,
    then the same tile of up rows, for t = 0 .. I / pair_rows - 1."""
    if gate.shape != up.shape or gate.dim() != 3 or gate.shape[1] % pair_rows:
        raise ValueError(f"gate {tuple(gate.shape)} / up {tuple(up.shape)}: not [E, I, D] "
                         f"pairs with I a multiple of {pair_rows}")
    E, I, D = gate.shape
    g = gate.reshape(E, I // pair_rows, 1, pair_rows, D)
    u = up.reshape(E, I // pair_rows, 1, pair_rows, D)
    return torch.cat([g, u], dim=2).reshape(E, 2 * I, D)


def split_gate_up(fused: torch.Tensor, pair_rows: int = 32):
    """The inverse of interleave_gate_up: (gate, up), each [E, I, D], contiguous."""
    if fused.dim() != 3 or fused.shape[1] % (2 * pair_rows):
        raise ValueError(f"fused {tuple(fused.shape)}: not [E, 2 I, D] with I a multiple of "
                         f"{pair_rows}")
    E, I2, D = fused.shape
    t = fused.reshape(E, I2 // (2 * pair_rows), 2, pair_rows, D)
    return (t[:, :, 0].reshape(E, I2 // 2, D).contiguous(),
            t[:, :, 1].reshape(E, I2 // 2, D).contiguous())


# --------------------------------------------------------------------------
# the checkpoint directory
# --------------------------------------------------------------------------

INDEX_NAME = "model.safetensors.index.json"


def _check_quantization(cfg: dict):
    q, qc = cfg.get("quantization"), cfg.get("quantization_config")
    if q is None or qc is None:
        raise CheckpointError("config.json needs both quantization and quantization_config")
    if q != qc:
        raise CheckpointError(f"quantization {q} != quantization_config {qc}")
    if q != NVFP4_QUANT:
        raise CheckpointError(f"quantization must be exactly {NVFP4_QUANT}, got {q}")


class LagunaCheckpoint:
    """A Laguna NVFP4 checkpoint directory, validated against the weight
    contract on open (index and shards; `check_inventory()` adds the full
    name / dtype / shape check)."""

    def __init__(self, directory: str):
        self.dir = directory
        try:
            with open(os.path.join(directory, "config.json")) as f:
                self.config = json.load(f)
        except FileNotFoundError:
            raise CheckpointError(f"{directory}: no config.json") from None
        _check_quantization(self.config)
        self.geometry = LagunaGeometry.from_config(self.config)
        try:
            with open(os.path.join(directory, INDEX_NAME)) as f:
                index = json.load(f)
        except FileNotFoundError:
            raise CheckpointError(f"{directory}: no {INDEX_NAME}") from None
        wm = index.get("weight_map")
        if not isinstance(wm, dict) or not wm:
            raise CheckpointError(f"{INDEX_NAME}: no weight_map")
        self.weight_map = {n: s for n, s in wm.items() if not n.endswith("rotary_emb.inv_freq")}
        shards = sorted(set(self.weight_map.values()))
        present = sorted(n for n in os.listdir(directory) if n.endswith(".safetensors"))
        missing = [s for s in shards if s not in present]
        if missing:
            raise CheckpointError(f"shards named by the index are missing: {missing}")
        extra = [s for s in present if s not in shards]
        if extra:
            raise CheckpointError(f"shards not named by the index: {extra}")
        self.shards = {}
        seen = {}
        for s in shards:
            f = SafetensorsFile(os.path.join(directory, s))
            names = {n for n in f.names() if not n.endswith("rotary_emb.inv_freq")}
            want = {n for n, sh in self.weight_map.items() if sh == s}
            if names != want:
                d1, d2 = sorted(want - names)[:3], sorted(names - want)[:3]
                raise CheckpointError(f"{s}: holds other tensors than the index assigns it "
                                      f"(missing {d1}, unassigned {d2})")
            for n in names:
                if n in seen:
                    raise CheckpointError(f"tensor {n} in both {seen[n]} and {s}")
                seen[n] = s
            self.shards[s] = f

    # ---- lookups ----
    def info(self, name):
        return self.shards[self.weight_map[name]].info(name)

    def tensor(self, name, device="cpu") -> torch.Tensor:
        if name not in self.weight_map:
            raise CheckpointError(f"no tensor {name}")
        return self.shards[self.weight_map[name]].tensor(name, device)

    def inventory(self):
        """(name, dtype, shape, shard) of every tensor, name order."""
        return sorted((n, *self.info(n), s) for n, s in self.weight_map.items())

    def check_inventory(self):
        """Names, dtypes and shapes equal to expected_inventory(geometry), and
        no `.biases` companion of a quantized projection."""
        have = {n: self.info(n) for n in self.weight_map}
        bad = [n for n in have if n.endswith(".biases")]
        if bad:
            raise CheckpointError(f"quantized projections carry no biases: {bad[:3]}")
        want = {n: (d, tuple(s)) for n, d, s in expected_inventory(self.geometry)}
        missing = sorted(set(want) - set(have))
        extra = sorted(set(have) - set(want))
        if missing or extra:
            raise CheckpointError(f"inventory differs: missing {missing[:3]} "
                                  f"({len(missing)}), unexpected {extra[:3]} ({len(extra)})")
        for n, (d, s) in want.items():
            if have[n] != (d, s):
                raise CheckpointError(f"{n}: {have[n][0]} {list(have[n][1])}, the contract "
                                      f"says {d} {list(s)}")

    # ---- sparse layers ----
    def sparse_layer(self, n: int, device="cpu") -> dict:
        """Layer n's MoE tensors in the kernels' layout (the stored one):
        routed / shared banks (gate_w, gate_s, up_w, up_s, down_w, down_s),
        router_w, router_b and norm_w (post_attention_layernorm, the norm in
        front of the block)."""
        if self.geometry.mlp_layer_types[n] != "sparse":
            raise CheckpointError(f"layer {n} is {self.geometry.mlp_layer_types[n]}, not sparse")
        p = f"model.layers.{n}.mlp"

        def bank(stem):
            out = {}
            for proj in ("gate", "up", "down"):
                out[f"{proj}_w"] = self.tensor(f"{stem}.{proj}_proj.weight", device)
                out[f"{proj}_s"] = self.tensor(f"{stem}.{proj}_proj.scales", device)
            return out

        shared = (bank(f"{p}.shared_expert") if self.geometry.moe.shared_inter else None)
        return dict(routed=bank(f"{p}.switch_mlp"), shared=shared,
                    router_w=self.tensor(f"{p}.gate.weight", device),
                    router_b=self.tensor(f"{p}.gate.e_score_correction_bias", device),
                    norm_w=self.tensor(f"model.layers.{n}.post_attention_layernorm.weight",
                                       device))

    def sparse_block(self, nv, n: int, device="cuda:0"):
        """(SparseMoeBlock, raw dict) for sparse layer n, as
        laguna.random_sparse_layer returns for a random-init layer."""
        raw = self.sparse_layer(n, device)
        m = self.geometry.moe
        block = nv.SparseMoeBlock(raw["routed"], raw["shared"], raw["router_w"], raw["router_b"],
                                  top_k=m.top_k, routed_scaling=m.routed_scaling,
                                  norm_topk_prob=m.norm_topk_prob)
        return block, raw


def laguna_xs_2_1_config() -> dict:
    """The config.json entries the geometry reads, for Laguna XS 2.1 (the
    contract's geometry, :82-87: hidden 2048, vocab 100352, 40 layers, head
    dimension 128, 8 KV heads, 48 query heads on the full-attention layers
    0, 4, ..., 36 and 64 on the sliding ones, dense intermediate 8192 at
    layer 0, 256 experts top-8, expert and shared intermediate 512)."""
    L = 40
    return {
        "hidden_size": 2048, "vocab_size": 100352, "num_hidden_layers": L, "head_dim": 128,
        "num_key_value_heads": 8, "num_attention_heads": 48,
        "num_attention_heads_per_layer": [48 if i % 4 == 0 else 64 for i in range(L)],
        "mlp_layer_types": ["dense"] + ["sparse"] * (L - 1), "intermediate_size": 8192,
        "moe_intermediate_size": 512, "shared_expert_intermediate_size": 512,
        "num_experts": 256, "num_experts_per_tok": 8, "moe_routed_scaling_factor": 2.5,
        "norm_topk_prob": True, "rms_norm_eps": 1e-6,
        "quantization": dict(NVFP4_QUANT), "quantization_config": dict(NVFP4_QUANT),
    }
