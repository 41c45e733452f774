"""DeepSeek-V3 FP8 checkpoint ingest: experts read from safetensors shards straight into an
expert arena (``cst_upload_expert``), the router and the shared expert alongside.

The reference reads a checkpoint through ``DeepseekModelLoader``
(server/deepseek_model_loader.py): the shard index ``model.safetensors.index.json``
(``_load_safetensors_index``, :104-122), the tensor names of one routed expert
(``deepseek_tensor_name``, :12-28) and their block scales ``<name>_scale_inv``
(``resolve_deepseek_scale_tensor``, :150-163), and the coordinator orders the six tensors
of each placed expert into a preload manifest (``build_preload_manifest``,
server/coordinator.py:413-488).  This module keeps those names, the index rules and the
manifest order; it reads the shards itself -- the safetensors layout is an 8-byte
little-endian header length, a JSON header of ``{name: {dtype, shape, data_offsets}}`` and
the raw tensor bytes -- memory-mapping each shard so a tensor's bytes go to the device
without a host copy.  No tensor is dequantized on the host: the E4M3 bytes and their fp32
``scale_inv`` grids are the device format (``cst_upload_expert`` relays them out).
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

# safetensors dtype tags this path reads
_DTYPES = {"F8_E4M3": np.uint8, "F32": np.float32, "BF16": np.uint16, "F16": np.float16}

# the six tensors of one expert in the reference's manifest order (coordinator.py:419-426):
# (bundle kind, projection, is scale, wire order)
BUNDLE_ORDER = (("w_up", "up_proj", False, 0), ("w_up_scale", "up_proj", True, 1),
                ("w_gate", "gate_proj", False, 2), ("w_gate_scale", "gate_proj", True, 3),
                ("w_down", "down_proj", False, 4), ("w_down_scale", "down_proj", True, 5))


def deepseek_tensor_name(layer_id: int, expert_id: int, tensor_kind: str) -> str:
    """Checkpoint name of a routed expert's weight (server/deepseek_model_loader.py:12-28)."""
    proj = {"w_up": "up_proj", "w_gate": "gate_proj", "w_down": "down_proj"}.get(str(tensor_kind))
    if proj is None:
        raise ValueError(f"unsupported tensor_kind: {tensor_kind}")
    return f"model.layers.{int(layer_id)}.mlp.experts.{int(expert_id)}.{proj}.weight"


class SafetensorsShard:
    """One ``.safetensors`` file: its header parsed once, tensors as memory-mapped numpy views."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        with self.path.open("rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
        if not isinstance(header, dict):
            raise ValueError(f"{self.path}: safetensors header is not an object")
        header.pop("__metadata__", None)
        self.header = header
        self.data_start = 8 + n
        self._map = np.memmap(self.path, dtype=np.uint8, mode="c")  # copy-on-write: the file stays untouched

    def __contains__(self, name: str) -> bool:
        return name in self.header

    def tensor(self, name: str) -> tuple[np.ndarray, str]:
        """(array, safetensors dtype tag); F8_E4M3 comes back as its uint8 codes."""
        meta = self.header.get(name)
        if meta is None:
            raise KeyError(f"{name} not in {self.path}")
        tag = meta["dtype"]
        if tag not in _DTYPES:
            raise TypeError(f"{name}: unsupported dtype {tag}")
        b, e = (int(v) for v in meta["data_offsets"])
        shape = tuple(int(v) for v in meta["shape"])
        raw = self._map[self.data_start + b:self.data_start + e]
        arr = raw.view(_DTYPES[tag])
        if arr.size != int(np.prod(shape, dtype=np.int64)):
            raise ValueError(f"{name}: {e - b} bytes do not hold shape {shape} of {tag}")
        return arr.reshape(shape), tag


@dataclass(frozen=True)
class TensorSpec:
    """One tensor of a preload bundle (server/coordinator.py:21-26)."""

    tensor_kind_name: str
    tensor_order: int
    tensor_name: str
    shard_path: str


@dataclass(frozen=True)
class BundleSpec:
    """The six tensors of one placed expert (server/coordinator.py:30-33)."""

    expert_id: int
    target: dict
    tensors: list


class DeepseekCheckpoint:
    """A DeepSeek-V3 checkpoint directory: ``config.json`` + ``model.safetensors.index.json`` + shards."""

    def __init__(self, model_root: str | Path):
        self.model_root = Path(model_root)
        self._weight_map = self._load_index(self.model_root)
        self._shards: dict[str, SafetensorsShard] = {}
        self._config = None

    @staticmethod
    def _load_index(model_root: Path) -> dict[str, str]:
        """``_load_safetensors_index`` (server/deepseek_model_loader.py:104-122): name -> shard path."""
        with (model_root / "model.safetensors.index.json").open("r", encoding="utf-8") as f:
            obj = json.load(f)
        weight_map = obj.get("weight_map")
        if not isinstance(weight_map, dict):
            raise ValueError("model.safetensors.index.json missing weight_map")
        out = {}
        for name, rel in weight_map.items():
            if not isinstance(name, str):
                raise ValueError("invalid tensor name in weight_map")
            if not isinstance(rel, str):
                raise ValueError(f"invalid shard path for tensor {name}")
            out[name] = str(model_root / rel)
        return out

    def weight_map(self) -> dict[str, str]:
        return self._weight_map

    def config(self) -> dict:
        if self._config is None:
            p = self.model_root / "config.json"
            if not p.exists():
                raise RuntimeError(f"config.json not found: {p}")
            obj = json.loads(p.read_text(encoding="utf-8"))
            if not isinstance(obj, dict):
                raise ValueError("config.json must decode to dict")
            self._config = obj
        return self._config

    def router_config(self) -> dict:
        """The router fields of ``config.json`` (server/deepseek_model_loader.py:66-81)."""
        c = self.config()
        return {"n_group": int(c["n_group"]), "topk_group": int(c["topk_group"]),
                "top_k": int(c["num_experts_per_tok"]), "norm_topk_prob": bool(c["norm_topk_prob"]),
                "routed_scaling_factor": float(c["routed_scaling_factor"]), "scoring_func": str(c["scoring_func"]),
                "topk_method": str(c["topk_method"]), "n_routed_experts": int(c["n_routed_experts"]),
                "hidden_size": int(c["hidden_size"])}

    # -- names ------------------------------------------------------------------------
    def resolve_tensor(self, tensor_name: str) -> tuple[str, str]:
        shard = self._weight_map.get(str(tensor_name))
        if shard is None:
            raise KeyError(f"tensor not found in index: {tensor_name}")
        return str(tensor_name), shard

    def resolve_deepseek_tensor(self, layer_id: int, expert_id: int, tensor_kind: str) -> tuple[str, str]:
        return self.resolve_tensor(deepseek_tensor_name(layer_id, expert_id, tensor_kind))

    def resolve_deepseek_scale_tensor(self, layer_id: int, expert_id: int, tensor_kind: str) -> tuple[str, str]:
        name, _ = self.resolve_deepseek_tensor(layer_id, expert_id, tensor_kind)
        return self.resolve_tensor(name + "_scale_inv")

    # -- tensors ----------------------------------------------------------------------
    def _shard(self, path: str) -> SafetensorsShard:
        if path not in self._shards:
            self._shards[path] = SafetensorsShard(path)
        return self._shards[path]

    def tensor(self, tensor_name: str) -> tuple[np.ndarray, str]:
        name, shard = self.resolve_tensor(tensor_name)
        return self._shard(shard).tensor(name)

    def _fp8_pair(self, weight_name: str) -> tuple[np.ndarray, np.ndarray]:
        w, tag = self.tensor(weight_name)
        if tag != "F8_E4M3":
            raise TypeError(f"{weight_name}: expected float8_e4m3fn, got {tag}")
        s, stag = self.tensor(weight_name + "_scale_inv")
        if stag != "F32":
            raise TypeError(f"{weight_name}_scale_inv: expected float32, got {stag}")
        return w, s

    def expert_bundle(self, layer_id: int, expert_id: int | None) -> dict:
        """The six upload tensors of routed expert ``expert_id`` (None: the shared expert) of a
        layer, as memory-mapped arrays in the upload format (uint8 E4M3 codes, fp32 scale_inv)."""
        if expert_id is None:
            base = f"model.layers.{int(layer_id)}.mlp.shared_experts"
        else:
            base = f"model.layers.{int(layer_id)}.mlp.experts.{int(expert_id)}"
        out = {}
        for kind, proj in (("w_up", "up_proj"), ("w_gate", "gate_proj"), ("w_down", "down_proj")):
            w, s = self._fp8_pair(f"{base}.{proj}.weight")
            out[kind], out[kind + "_scale"] = w, s
        return out

    def router_tensors(self, layer_id: int) -> tuple[np.ndarray, np.ndarray]:
        """(gate weight [E, H], e_score_correction_bias [E]) as fp32
        (``load_router_tensors_fp32``, server/deepseek_model_loader.py:283-292)."""
        def f32(name):
            a, tag = self.tensor(name)
            if tag == "F32":
                return np.array(a, dtype=np.float32)
            if tag == "BF16":
                return (a.astype(np.uint32) << 16).view(np.float32)
            if tag == "F16":
                return a.astype(np.float32)
            raise TypeError(f"{name}: unsupported router dtype {tag}")

        base = f"model.layers.{int(layer_id)}.mlp.gate"
        return f32(base + ".weight"), f32(base + ".e_score_correction_bias")

    # -- preload ----------------------------------------------------------------------
    def build_preload_manifest(self, placements, experts_per_layer: int = 256) -> list[BundleSpec]:
        """One bundle per placement ``{"expert_id": global id, "host", "control_port", ...}``,
        its six tensors in the wire order, bundles sorted by (host, control_port, expert_id)
        -- ``build_preload_manifest`` (server/coordinator.py:413-488)."""
        manifest = []
        for target in placements:
            gid = int(target["expert_id"])
            layer, local = gid // experts_per_layer, gid % experts_per_layer
            specs = []
            for kind, proj, is_scale, order in BUNDLE_ORDER:
                base_kind = kind[:-len("_scale")] if is_scale else kind
                resolve = self.resolve_deepseek_scale_tensor if is_scale else self.resolve_deepseek_tensor
                name, shard = resolve(layer, local, base_kind)
                specs.append(TensorSpec(kind, order, name, str(shard)))
            manifest.append(BundleSpec(gid, target, specs))
        manifest.sort(key=lambda b: (str(b.target["host"]), int(b.target["control_port"]), int(b.expert_id)))
        return manifest

    def upload_layer(self, ctx, layer_id: int, experts=None, *, shared: bool = True,
                     first_slot: int = 0) -> dict[int, int]:
        """Upload routed experts ``experts`` (default: all of the layer) and the shared expert
        of one layer into consecutive slots of ``ctx`` (an ``ExpertContext``) from the shards.
        Returns {router expert id (-1 = shared): slot}."""
        if experts is None:
            experts = range(int(self.config().get("n_routed_experts", ctx.cfg.n_routed_experts)))
        placed = {}
        slot = int(first_slot)
        for e in list(experts) + ([None] if shared else []):
            b = self.expert_bundle(layer_id, e)
            eid = -1 if e is None else int(e)
            ctx.upload_expert(slot, eid, b["w_up"], b["w_up_scale"], b["w_gate"], b["w_gate_scale"], b["w_down"],
                              b["w_down_scale"])
            placed[eid] = slot
            slot += 1
        return placed


__all__ = ["deepseek_tensor_name", "SafetensorsShard", "DeepseekCheckpoint", "BundleSpec", "TensorSpec",
           "BUNDLE_ORDER"]
