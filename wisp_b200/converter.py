"""Int4 expert format: quantiser, expert ``.bin`` writer and model-directory writer.

This is the offline side of the MoE path: it produces the bytes the CUDA kernels
consume.  The format is WISP's, bit for bit, so a directory written here loads in
the reference engine and vice versa.

Quantiser (restates ``wisp/converter/quantizer.py:46-86``; the arithmetic has to be
identical because the oracle and the GPU path are compared on the same codes):

* groups of ``group_size`` consecutive row-major elements (the tail group is padded
  by repeating the last element);
* ``zero = (max + min) / 2`` and ``scale = max((max - min) / 15, 1e-8)`` in fp32;
* ``q = clamp(round_half_even((x - zero) / scale) + 8, 0, 15)``;
* two codes per byte, even element in the low nibble;
* scale and zero are stored as fp16, so every consumer dequantises with the
  fp16-rounded values: ``w = (q - 8) * scale16 + zero16``.

Expert blob (restates ``wisp/converter/partitioner.py:11-26,56-89``; the layout is
the on-disk contract with ``csrc/core/wisp_engine.c:268-303``): a 120-byte header
``<6I`` (magic, version, layer, expert, group_size, n_mats=3) then three ``<2I3Q``
matrix records (rows, cols, packed, scales, zeros byte counts), then per matrix
``packed | scales | zeros`` in gate, up, down order.

The functions accept CPU or CUDA tensors; the same ops give the same bits on both
devices (IEEE division, round-half-even, fp16 round-to-nearest-even).
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

EXPERT_MAGIC = 0x57455850
EXPERT_VERSION = 1
HEADER = struct.Struct("<6I")
MAT_RECORD = struct.Struct("<2I3Q")
HEADER_BYTES = HEADER.size + 3 * MAT_RECORD.size  # 120
MAT_ORDER = ("gate", "up", "down")


@dataclass
class QMat:
    """One int4-quantised matrix: packed codes plus fp16 scale and zero per group."""

    packed: torch.Tensor  # uint8 [ceil(n/2)]
    scales: torch.Tensor  # fp16 [n_groups]
    zeros: torch.Tensor   # fp16 [n_groups]
    rows: int
    cols: int
    group_size: int

    def section_bytes(self) -> tuple[int, int, int]:
        return (self.packed.numel(), self.scales.numel() * 2, self.zeros.numel() * 2)


def quantize_int4(weight: torch.Tensor, group_size: int = 64) -> QMat:
    """Group-wise asymmetric int4 quantisation of a 2-D weight (see module doc)."""
    if weight.dim() != 2:
        raise ValueError(f"quantize_int4 expects a 2-D weight, got shape {tuple(weight.shape)}")
    if group_size <= 0:
        raise ValueError(f"group_size must be positive, got {group_size}")
    rows, cols = (int(s) for s in weight.shape)
    v = weight.detach().to(torch.float32).reshape(-1)
    n = v.numel()
    n_groups = -(-n // group_size)
    pad = n_groups * group_size - n
    if pad:
        v = torch.cat([v, v[-1:].expand(pad)])
    g = v.view(n_groups, group_size)
    hi = g.amax(dim=1)
    lo = g.amin(dim=1)
    zero = (hi + lo) / 2.0
    scale = torch.clamp((hi - lo) / 15.0, min=1e-8)
    codes = torch.round((g - zero[:, None]) / scale[:, None]) + 8
    codes = codes.clamp_(0, 15).to(torch.uint8).reshape(-1)[:n]
    if n % 2:
        codes = torch.cat([codes, codes.new_zeros(1)])
    packed = (codes[0::2] | (codes[1::2] << 4)).contiguous()
    return QMat(packed, scale.to(torch.float16).contiguous(), zero.to(torch.float16).contiguous(),
                rows, cols, group_size)


def dequantize_int4(q: QMat) -> torch.Tensor:
    """fp32 ``[rows, cols]`` weight the kernels multiply by: ``(code-8)*scale16 + zero16``."""
    n = q.rows * q.cols
    codes = torch.stack([q.packed & 0x0F, q.packed >> 4], dim=1).reshape(-1)[:n].to(torch.float32)
    gi = torch.arange(n, device=q.packed.device) // q.group_size
    w = (codes - 8.0) * q.scales.to(torch.float32)[gi] + q.zeros.to(torch.float32)[gi]
    return w.view(q.rows, q.cols)


def expert_blob(layer: int, expert: int, mats: dict[str, QMat]) -> bytes:
    """Serialise gate/up/down into one expert ``.bin`` blob."""
    missing = [m for m in MAT_ORDER if m not in mats]
    if missing:
        raise ValueError(f"expert L{layer}/E{expert} incomplete: missing {missing}")
    ordered = [mats[m] for m in MAT_ORDER]
    parts = [HEADER.pack(EXPERT_MAGIC, EXPERT_VERSION, layer, expert, ordered[0].group_size, 3)]
    parts += [MAT_RECORD.pack(q.rows, q.cols, *q.section_bytes()) for q in ordered]
    for q in ordered:
        parts += [q.packed.cpu().numpy().tobytes(), q.scales.cpu().numpy().tobytes(),
                  q.zeros.cpu().numpy().tobytes()]
    return b"".join(parts)


def parse_blob_header(blob: bytes | memoryview) -> dict:
    """Header fields and section offsets of an expert blob (raises on corruption)."""
    if len(blob) < HEADER_BYTES:
        raise ValueError(f"expert blob too small: {len(blob)} bytes")
    magic, ver, layer, expert, gs, nm = HEADER.unpack_from(blob, 0)
    if magic != EXPERT_MAGIC or ver not in (EXPERT_VERSION, TILED_VERSION) or nm != 3:
        raise ValueError(f"expert blob corrupt: magic={magic:08x} version={ver} n_mats={nm}")
    off = HEADER_BYTES
    mats = []
    for i in range(3):
        r, c, pb, sb, zb = MAT_RECORD.unpack_from(blob, HEADER.size + i * MAT_RECORD.size)
        mats.append(dict(rows=r, cols=c, packed_off=off, scales_off=off + pb,
                         zeros_off=off + pb + sb, packed_bytes=pb, scales_bytes=sb, zeros_bytes=zb))
        off += pb + sb + zb
    if off > len(blob):
        raise ValueError(f"expert blob truncated: needs {off}, have {len(blob)}")
    return dict(layer=layer, expert=expert, group_size=gs, mats=mats, total_bytes=off,
                tiled=ver == TILED_VERSION)


# --------------------------------------------------------------------------------------
# Tiled device layout (version 2): the order the CUDA kernels stream.  Each matrix keeps
# its region; inside it every 8-row block is contiguous: for each quant group g the
# gs/2 code bytes of the block's 8 rows, then for each g the 8 rows' (scale, zero) fp16
# pairs.  These numpy restatements are the test-side checkers of wisp_expert_tile.
# --------------------------------------------------------------------------------------
TILED_VERSION = 2


def _tile_matrix(region: np.ndarray, rows: int, cols: int, gs: int) -> np.ndarray:
    G = cols // gs
    pb, sb = rows * cols // 2, rows * G * 2
    codes = region[:pb].reshape(rows // 8, 8, G, gs // 2).transpose(0, 2, 1, 3)
    sc = region[pb:pb + sb].view(np.uint16).reshape(rows // 8, 8, G)
    ze = region[pb + sb:pb + 2 * sb].view(np.uint16).reshape(rows // 8, 8, G)
    sz = np.stack([sc, ze], axis=-1).transpose(0, 2, 1, 3)  # [block][g][row][s, z]
    blocks = np.concatenate([codes.reshape(rows // 8, -1),
                             np.ascontiguousarray(sz).view(np.uint8).reshape(rows // 8, -1)],
                            axis=1)
    return blocks.reshape(-1)


def _untile_matrix(region: np.ndarray, rows: int, cols: int, gs: int) -> np.ndarray:
    G = cols // gs
    blocks = region.reshape(rows // 8, 4 * cols + 32 * G)
    codes = blocks[:, :4 * cols].reshape(rows // 8, G, 8, gs // 2).transpose(0, 2, 1, 3)
    sz = np.ascontiguousarray(blocks[:, 4 * cols:]).view(np.uint16).reshape(rows // 8, G, 8, 2)
    sc = sz[..., 0].transpose(0, 2, 1)
    ze = sz[..., 1].transpose(0, 2, 1)
    return np.concatenate([codes.reshape(-1), np.ascontiguousarray(sc).view(np.uint8).reshape(-1),
                           np.ascontiguousarray(ze).view(np.uint8).reshape(-1)])


def _retile(blob, fn, version: int) -> np.ndarray:
    b = np.frombuffer(bytes(blob), dtype=np.uint8).copy()
    h = parse_blob_header(b.tobytes()[:HEADER_BYTES] + b"\0" * (len(b) - HEADER_BYTES))
    for m in h["mats"]:
        lo, hi = m["packed_off"], m["zeros_off"] + m["zeros_bytes"]
        b[lo:hi] = fn(b[lo:hi], m["rows"], m["cols"], h["group_size"])
    b[4:8] = np.frombuffer(struct.pack("<I", version), dtype=np.uint8)
    return b


def tile_blob(blob) -> np.ndarray:
    """A ``.bin`` blob rewritten into the tiled device layout (header version 2)."""
    return _retile(blob, _tile_matrix, TILED_VERSION)


def untile_blob(blob) -> np.ndarray:
    """The ``.bin`` blob a tiled blob was made from."""
    return _retile(blob, _untile_matrix, EXPERT_VERSION)


def qmats_from_blob(blob) -> dict[str, QMat]:
    """The three matrices of a ``.bin`` blob (bytes or uint8 array) as QMats."""
    b = bytes(blob)
    h = parse_blob_header(b)
    if h["tiled"]:
        raise ValueError("qmats_from_blob wants a .bin blob (untile it first)")
    out = {}
    for name, m in zip(MAT_ORDER, h["mats"]):
        def sect(off, n, dt):
            return torch.frombuffer(bytearray(b[off:off + n]), dtype=dt)
        out[name] = QMat(sect(m["packed_off"], m["packed_bytes"], torch.uint8),
                         sect(m["scales_off"], m["scales_bytes"], torch.float16),
                         sect(m["zeros_off"], m["zeros_bytes"], torch.float16),
                         m["rows"], m["cols"], h["group_size"])
    return out


def expert_filename(layer: int, expert: int) -> str:
    return f"L{layer:03d}_E{expert:05d}.bin"


# --------------------------------------------------------------------------------------
# Seeded synthetic models (the benchmark's and the tests' inputs).
# --------------------------------------------------------------------------------------

@dataclass
class MoEShape:
    hidden: int
    inter: int
    n_experts: int
    top_k: int
    group_size: int = 64
    n_layers: int = 1
    shared_inter: int = 0      # 0 = no shared expert
    rms_eps: float = 1e-5


MIXTRAL = MoEShape(hidden=4096, inter=14336, n_experts=8, top_k=2)
DEEPSEEK = MoEShape(hidden=7168, inter=2048, n_experts=256, top_k=8, shared_inter=2048)


def expert_seed(seed: int, layer: int, expert: int, mat: int, n_experts: int) -> int:
    """Per-matrix seed: ``seed + ((layer * E + expert) * 3 + mat)``."""
    return seed + ((layer * n_experts + expert) * 3 + mat)


def _normal(shape, std: float, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


def make_expert(shape: MoEShape, layer: int, expert: int, seed: int, device="cpu",
                std: float = 0.02) -> dict[str, QMat]:
    """Gate/up ``[I, H]`` and down ``[H, I]`` drawn N(0, std) and quantised."""
    dims = {"gate": (shape.inter, shape.hidden), "up": (shape.inter, shape.hidden),
            "down": (shape.hidden, shape.inter)}
    out = {}
    for m, name in enumerate(MAT_ORDER):
        w = _normal(dims[name], std, expert_seed(seed, layer, expert, m, shape.n_experts), device)
        out[name] = quantize_int4(w, shape.group_size)
    return out


def make_shared_expert(shape: MoEShape, layer: int, seed: int, device="cpu",
                       std: float = 0.02) -> dict[str, QMat]:
    """The always-on shared expert, quantised the same way (seed offset past the routed ones)."""
    s = MoEShape(shape.hidden, shape.shared_inter, shape.n_experts + 1, shape.top_k, shape.group_size)
    return make_expert(s, layer, shape.n_experts, seed, device, std)


def make_router(shape: MoEShape, layer: int, seed: int, device="cpu", std: float = 0.02) -> torch.Tensor:
    """fp16 router ``[E, H]`` drawn N(0, std)."""
    return _normal((shape.n_experts, shape.hidden), std, seed + 7_000_000 + layer, device).to(torch.float16)


def zipf_router_bias(shape: MoEShape, s: float = 1.1, scale: float = 1.0) -> torch.Tensor:
    """fp16 router bias that skews softmax popularity towards Zipf(s): ``b_e = -s*log(e+1)``.

    Expert ``e`` gets a logit offset proportional to ``log(1/(e+1)^s)``, so its softmax
    mass follows the Zipf law before the data-dependent part of the logits is added.
    """
    e = torch.arange(shape.n_experts, dtype=torch.float32)
    return (-s * scale * torch.log(e + 1.0)).to(torch.float16)


def make_input(shape: MoEShape, tokens: int, seed: int, device="cpu") -> torch.Tensor:
    """Hidden states: fp16 N(0,1) upcast to fp32 (the block consumes fp32)."""
    return _normal((tokens, shape.hidden), 1.0, seed + 9_000_000, device).to(torch.float16).float()


def _safetensors_bytes(tensors: dict[str, torch.Tensor]) -> bytes:
    """Minimal safetensors serialiser (fp16 only, which is all the dense file holds)."""
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().to(torch.float16).contiguous().cpu()
        b = t.numpy().tobytes()
        header[name] = {"dtype": "F16", "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * (-len(hj) % 8)
    return struct.pack("<Q", len(hj)) + hj + b"".join(blobs)


def make_dense_ffn(hidden: int, inter: int, layer: int, seed: int, tag: int,
                   std: float = 0.02) -> dict[str, torch.Tensor]:
    """fp16 SwiGLU weights (gate/up ``[inter, hidden]``, down ``[hidden, inter]``) drawn
    N(0, std) and rounded to fp16, the form the reference converter stores shared
    experts and dense-MLP layers in (real-valued, not int4-representable).  ``tag``
    separates the shared expert (1) from a dense-MLP layer (2)."""
    dims = {"gate": (inter, hidden), "up": (inter, hidden), "down": (hidden, inter)}
    return {name: _normal(dims[name], std, seed + 8_000_000 + (layer * 3 + m) * 4 + tag,
                          "cpu").half()
            for m, name in enumerate(MAT_ORDER)}


def write_model_dir(path: str | Path, shape: MoEShape, seed: int, *, router_bias: bool = False,
                    zipf_s: float | None = None, shared_int4: bool = True, vocab: int = 16,
                    shared_form: str = "int4", dense_layers=(), dense_inter: int = 0,
                    missing=(), attention: dict | None = None) -> Path:
    """Write a converted-model directory (manifest, dense safetensors, expert blobs).

    The dense file carries what the reference loader requires (``embed_tokens``,
    ``final_norm``, ``lm_head``, per-layer ``input_norm``/``post_norm``/``attn.o_proj``)
    plus the router.  Norm weights are ones.  When the shape has a shared expert:

    * ``shared_form="int4"``: it is quantised like a routed expert and stored
      fp16-dense under ``layers.i.shared.*`` as the dequantised int4 weights (the
      reference runs shared experts dense) and, with ``shared_int4``, also as an int4
      blob ``experts/L{layer}_shared.bin`` that this engine prefers;
    * ``shared_form="fp16"``: real-valued fp16 weights under ``layers.i.shared.*``
      only (``make_dense_ffn``), as the reference converter writes a checkpoint's
      shared expert.

    ``dense_layers``: layers written without a router whose FFN is an fp16-dense
    SwiGLU of ``dense_inter`` rows under ``layers.i.shared.*`` (the reference's
    dense-MLP layers).  ``missing``: (layer, expert) pairs whose blob is not written.
    ``attention``: ``{"n_heads", "n_kv_heads", "rope_theta", "max_pos"}`` writes a GQA
    attention block per layer (``attn.{q,k,v,o}_proj`` seeded normal, ``input_norm``
    near 1) so the directory serves the whole decoder step; without it the attention
    tensors are the loader's minimum (``attn.o_proj`` only).
    """
    root = Path(path)
    (root / "experts").mkdir(parents=True, exist_ok=True)
    (root / "dense").mkdir(parents=True, exist_ok=True)
    H = shape.hidden
    dense: dict[str, torch.Tensor] = {
        "embed_tokens": _normal((vocab, H), 0.02, seed + 1, "cpu").half(),
        "final_norm": torch.ones(H, dtype=torch.float16),
        "lm_head": _normal((vocab, H), 0.02, seed + 2, "cpu").half(),
    }
    blob_bytes = 0
    missing = {tuple(m) for m in missing}
    for layer in range(shape.n_layers):
        if attention:
            nh, nkv = attention["n_heads"], attention["n_kv_heads"]
            hd = H // nh
            base = seed + 1000 * (layer + 1)
            dense[f"layers.{layer}.input_norm"] = (
                1.0 + _normal((H,), 0.1, base, "cpu")).half()
            dense[f"layers.{layer}.post_norm"] = (
                1.0 + _normal((H,), 0.1, base + 1, "cpu")).half()
            dense[f"layers.{layer}.attn.q_proj"] = _normal((nh * hd, H), 0.5 / H ** 0.5, base + 2,
                                                           "cpu").half()
            dense[f"layers.{layer}.attn.k_proj"] = _normal((nkv * hd, H), 0.5 / H ** 0.5,
                                                           base + 3, "cpu").half()
            dense[f"layers.{layer}.attn.v_proj"] = _normal((nkv * hd, H), 1.0 / H ** 0.5,
                                                           base + 4, "cpu").half()
            dense[f"layers.{layer}.attn.o_proj"] = _normal((H, nh * hd), 0.5 / (nh * hd) ** 0.5,
                                                           base + 5, "cpu").half()
        else:
            dense[f"layers.{layer}.input_norm"] = torch.ones(H, dtype=torch.float16)
            dense[f"layers.{layer}.post_norm"] = torch.ones(H, dtype=torch.float16)
            dense[f"layers.{layer}.attn.o_proj"] = torch.zeros(1, 1, dtype=torch.float16)
        if layer in dense_layers:
            for name, t in make_dense_ffn(H, dense_inter, layer, seed, 2).items():
                dense[f"layers.{layer}.shared.{name}"] = t
            continue
        dense[f"layers.{layer}.router"] = make_router(shape, layer, seed)
        if router_bias or zipf_s is not None:
            dense[f"layers.{layer}.router_bias"] = (
                zipf_router_bias(shape, zipf_s) if zipf_s is not None
                else _normal((shape.n_experts,), 0.5, seed + 3 + layer, "cpu").half())
        for e in range(shape.n_experts):
            blob = expert_blob(layer, e, make_expert(shape, layer, e, seed))
            blob_bytes = max(blob_bytes, len(blob))
            if (layer, e) not in missing:
                (root / "experts" / expert_filename(layer, e)).write_bytes(blob)
        if shape.shared_inter and shared_form == "fp16":
            for name, t in make_dense_ffn(H, shape.shared_inter, layer, seed, 1).items():
                dense[f"layers.{layer}.shared.{name}"] = t
        elif shape.shared_inter:
            sh = make_shared_expert(shape, layer, seed)
            for name in MAT_ORDER:
                dense[f"layers.{layer}.shared.{name}"] = dequantize_int4(sh[name]).half()
            if shared_int4:
                (root / "experts" / f"L{layer:03d}_shared.bin").write_bytes(
                    expert_blob(layer, 0xFFFF, sh))
    (root / "dense" / "model_dense.safetensors").write_bytes(_safetensors_bytes(dense))
    manifest = {
        "wisp_version": "2.0.0",
        "model_family": "synthetic-moe",
        "model_name": "synthetic-moe",
        "architecture": {
            "attention_type": "GQA",
            "num_layers": shape.n_layers,
            "num_experts_per_layer": shape.n_experts,
            "num_shared_experts": 1 if shape.shared_inter else 0,
            "top_k_routing": shape.top_k,
            "hidden_size": H,
            "vocab_size": vocab,
            "moe_intermediate_size": shape.inter,
            "intermediate_size": shape.shared_inter or shape.inter,
            "num_attention_heads": attention["n_heads"] if attention else 1,
            "num_kv_heads": attention["n_kv_heads"] if attention else 1,
            "rope_theta": attention.get("rope_theta", 10000.0) if attention else 10000.0,
            "rms_norm_eps": shape.rms_eps,
            "max_position_embeddings": attention.get("max_pos", 256) if attention else 16,
        },
        "quantization": {"weight_dtype": "int4", "scale_dtype": "float16",
                         "zero_dtype": "float16", "group_size": shape.group_size},
        "performance": {"expert_size_bytes": blob_bytes},
        "files": {"dense_layers": "dense/model_dense.safetensors", "expert_dir": "experts/",
                  "expert_naming": "L{layer:03d}_E{expert:05d}.bin"},
        "seed": seed,
    }
    (root / "manifest.json").write_text(json.dumps(manifest, indent=2))
    return root
