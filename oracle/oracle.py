"""CPU oracle of the routed-MoE chain (TEST INFRASTRUCTURE, never the product).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
import this module. It restates the reference's algorithm for each step:

  * bit-exact parts in C (oracle/mm_oracle.c, loaded through ctypes): the router
    GEMV in the kernel's summation order, deterministic scores, top-k with bias,
    the route record, MXFP8 quantization, the slot-order combine;
  * the dense expert MLP by dequantize -> fp32 matmul (torch on the CPU), in two
    numerics: "exact" (bf16 input, fp32 throughout: BASELINE's tolerance
    reference) and "kernel" (the inputs of both GEMMs passed through the same
    MXFP4 activation terms the kernels use).

MXFP4 codec: OCP MX E2M1 (+-{0, .5, 1, 1.5, 2, 3, 4, 6}), byte = element 2j in the
low nibble and 2j+1 in the high nibble; E8M0 scale 2^(byte - 127) per 32
elements along K (glm5_3/sm103/moe/api.py:39-53, route_quant.cuh:1-15).
Expert MLP: gemm1.cu:6-7 + epilogue :656-1000 (clamped SwiGLU: up in [-L, L],
gate <= L, h = up * gate * sigmoid(gate)), gemm2.cu:6-7. Combine:
all_reduce_mhc.py:528-640; cross-rank sum: all_reduce_mhc.py:955-977.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import c_float, c_int, c_uint8, c_void_p
from typing import Optional

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_route.so")

E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)

_lib = None


def reference_root() -> Optional[str]:
    """The reference checkout named by MM_REFERENCE_ROOT (the directory holding
    sgl_nvidia_mega/), or None when unset or absent."""
    root = os.environ.get("MM_REFERENCE_ROOT", "")
    return root if root and os.path.isdir(os.path.join(root, "sgl_nvidia_mega")) else None


def build(ref: bool = False) -> None:
    """Compile the C oracle (and, with ``ref`` and MM_REFERENCE_ROOT naming a
    reference checkout, the reference's route kernels for the CPU)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    root = reference_root()
    if ref and root is not None:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={root}"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(os.path.join(HERE, "mm_oracle.c")):
            build()
        h = ctypes.CDLL(LIB)
        h.or_det_exp.restype = c_float
        h.or_det_exp.argtypes = [c_float]
        h.or_sigmoid.restype = c_float
        h.or_sigmoid.argtypes = [c_float]
        h.or_e4m3.restype = c_uint8
        h.or_e4m3.argtypes = [c_float]
        h.or_nv4_scale_code.restype = c_uint8
        h.or_nv4_scale_code.argtypes = [c_float, c_float]
        h.or_route_words.restype = c_int
        h.or_gate_topk.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float, c_int, c_int, c_int,
                                   c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_int64]
        _lib = h
    return _lib


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(c_void_p)


# --------------------------------------------------------------------- bit-exact steps
def router_gemv(x_bf16: np.ndarray, w_bf16: np.ndarray) -> np.ndarray:
    """x, w as uint16 bf16 bit patterns [T, H], [E, H] -> fp32 logits [T, E]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    T, H = x.shape
    E = w.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    lib().or_router_gemv(_p(x), _p(w), _p(out), T, E, H)
    return out


# routing weight rules: "scaled_bf16" is GLM-5.3's bf16(scale * s / (sum + eps))
# with the butterfly-order sum (glm5_3/sm103/moe/routing.py:3-11)
RENORM = {"none": 0, "sum": 1, "scaled_bf16": 2}


def gate_topk(logits: np.ndarray, bias: Optional[np.ndarray], top_k: int, *, score: str = "sigmoid",
              renormalize=True, scale: float = 1.0, eps: float = 0.0, num_valid: Optional[int] = None,
              bias_alt: Optional[np.ndarray] = None, input_ids: Optional[np.ndarray] = None,
              alt_token_id: int = -1):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    ba = None if bias_alt is None else np.ascontiguousarray(bias_alt, dtype=np.float32)
    tok = None if input_ids is None else np.ascontiguousarray(input_ids, dtype=np.int64)
    w = np.empty((T, top_k), dtype=np.float32)
    ids = np.empty((T, top_k), dtype=np.int32)
    sf = {"sigmoid": 0, "softmax": 1, "sqrtsoftplus": 2}[score]
    rn = RENORM[renormalize] if isinstance(renormalize, str) else int(bool(renormalize))
    lib().or_gate_topk(_p(logits), _p(b), T if num_valid is None else int(num_valid), sf, rn,
                       c_float(scale), c_float(eps), T, E, top_k, _p(w), _p(ids), _p(ba), _p(tok),
                       ctypes.c_int64(alt_token_id))
    return w, ids


def route_words(T: int, K: int, experts: int) -> int:
    return int(lib().or_route_words(T, K, experts))


def route(ids: np.ndarray, experts: int, offset: int = 0):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    perm = np.empty((T, K), dtype=np.int32)
    rec = np.empty(route_words(T, K, experts), dtype=np.int32)
    lib().or_route(_p(ids), _p(perm), _p(rec), T, K, experts, offset)
    return perm, rec


def mxfp8_quant(v: np.ndarray, terms: int = 2):
    """fp32 [..., K] (K % 32 == 0) -> (q_hi, q_lo, s_hi, s_lo) uint8 arrays."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    nb = v.size // 32
    qh = np.zeros(v.shape, dtype=np.uint8)
    ql = np.zeros(v.shape, dtype=np.uint8)
    sh = np.zeros(v.shape[:-1] + (v.shape[-1] // 32,), dtype=np.uint8)
    sl = np.zeros_like(sh)
    lib().or_mxfp8_quant(_p(v), nb, terms, _p(qh), _p(ql), _p(sh), _p(sl))
    return qh, ql, sh, sl


def e4m3_table() -> np.ndarray:
    h = lib()
    h.or_e4m3_value.restype = c_float
    h.or_e4m3_value.argtypes = [c_uint8]
    return np.array([h.or_e4m3_value(i) for i in range(256)], dtype=np.float32)


_E4M3 = None


def mxfp8_dequant(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    global _E4M3
    if _E4M3 is None:
        _E4M3 = e4m3_table()
    vals = _E4M3[q]
    scale = np.exp2(s.astype(np.float32) - 127.0).astype(np.float32)
    return (vals.reshape(*s.shape, 32) * scale[..., None]).reshape(q.shape)


def mxfp8_roundtrip(v: np.ndarray, terms: int = 1) -> np.ndarray:
    """v through MXFP8 (the reference kernels' activation numerics; terms 2 adds
    the MXFP8 residual term)."""
    qh, ql, sh, sl = mxfp8_quant(v, terms)
    out = mxfp8_dequant(qh, sh)
    if terms > 1:
        out = out + mxfp8_dequant(ql, sl)
    return out


def fp4_quant(v: np.ndarray, terms: int = 3):
    """fp32 [..., K] -> (codes u8 [terms, ..., K/2], scales u8 [terms, ..., K/32]):
    the kernels' MXFP4 activation terms."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    nb = v.size // 32
    q = np.zeros((terms, nb * 16), dtype=np.uint8)
    s = np.zeros((terms, nb), dtype=np.uint8)
    lib().or_fp4_quant(_p(v), nb, terms, _p(q), _p(s))
    lead = v.shape[:-1]
    return q.reshape(terms, *lead, v.shape[-1] // 2), s.reshape(terms, *lead, v.shape[-1] // 32)


def fp4_dequant(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """Sum of the MXFP4 terms (exact)."""
    lo = E2M1[q & 0x0F]
    hi = E2M1[q >> 4]
    vals = np.stack([lo, hi], axis=-1).reshape(*q.shape[:-1], q.shape[-1] * 2)
    scale = np.exp2(s.astype(np.float32) - 127.0).astype(np.float32)
    out = (vals.reshape(*s.shape, 32) * scale[..., None]).reshape(vals.shape)
    return out.sum(axis=0)


def act_roundtrip(v: np.ndarray, terms: int = 3, fmt: str = "mxfp4", input_scale: float = 1.0) -> np.ndarray:
    """The value the kernels multiply in place of activation v: the sum of its
    MXFP4 terms, or of its NVFP4 terms under the static input scale."""
    if fmt == "nvfp4":
        q, s = nvfp4_quant(v, terms, input_scale)
        return nvfp4_dequant(q, s, input_scale)
    q, s = fp4_quant(v, terms)
    return fp4_dequant(q, s).astype(np.float32)


_E4M3_LUT = None


def e4m3_lut() -> np.ndarray:
    """fp32 value of every E4M3 byte (exact decode)."""
    global _E4M3_LUT
    if _E4M3_LUT is None:
        _E4M3_LUT = e4m3_table()
    return _E4M3_LUT


def nvfp4_quant(v: np.ndarray, terms: int, input_scale: float):
    """fp32 [..., K] -> (codes u8 [terms, ..., K/2], E4M3 scales u8 [terms, ..., K/16]):
    the kernels' NVFP4 activation terms under global scale gs = 1 / input_scale."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    nb = v.size // 16
    q = np.zeros((terms, nb * 8), dtype=np.uint8)
    s = np.zeros((terms, nb), dtype=np.uint8)
    gs = np.float32(1.0) / np.float32(input_scale)
    lib().or_nvfp4_quant(_p(v), nb, terms, c_float(gs), c_float(input_scale), _p(q), _p(s))
    lead = v.shape[:-1]
    return q.reshape(terms, *lead, v.shape[-1] // 2), s.reshape(terms, *lead, v.shape[-1] // 16)


def nvfp4_dequant(q: np.ndarray, s: np.ndarray, input_scale: float) -> np.ndarray:
    """Sum over terms of e2m1 * e4m3 * input_scale (float64, returned as fp32)."""
    lo = E2M1[q & 0x0F].astype(np.float64)
    hi = E2M1[q >> 4].astype(np.float64)
    vals = np.stack([lo, hi], axis=-1).reshape(*q.shape[:-1], q.shape[-1] * 2)
    sc = e4m3_lut()[s].astype(np.float64)
    out = (vals.reshape(*s.shape, 16) * sc[..., None]).reshape(vals.shape)
    return (out.sum(axis=0) * float(input_scale)).astype(np.float32)


def dequant_nvfp4(codes: torch.Tensor, scales: torch.Tensor, scale_2: float) -> torch.Tensor:
    """u8 [..., K/2] codes + u8 [..., K/16] E4M3 + fp32 second-level scale ->
    fp32 [..., K] (ModelOpt NVFP4: w = e2m1 * e4m3 * scale_2). e2m1 * e4m3 is
    exact in fp32 (at most 5 significant bits), so the one rounding is that of
    the product with scale_2, as in an exact evaluation rounded to fp32."""
    lut = torch.from_numpy(E2M1)
    lo = lut[(codes & 0x0F).long()]
    hi = lut[(codes >> 4).long()]
    vals = torch.stack([lo, hi], dim=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)
    sc = torch.from_numpy(e4m3_lut())[scales.long()]
    out = (vals.reshape(*scales.shape, 16) * sc[..., None]).reshape(vals.shape)
    return out * torch.tensor(float(scale_2), dtype=torch.float32)


def finalize(rows_bf16: np.ndarray, weights: np.ndarray, permuted: np.ndarray,
             shared_bf16: Optional[np.ndarray]) -> np.ndarray:
    rows = np.ascontiguousarray(rows_bf16, dtype=np.uint16)
    w = np.ascontiguousarray(weights, dtype=np.float32)
    perm = np.ascontiguousarray(permuted, dtype=np.int32)
    sh = None if shared_bf16 is None else np.ascontiguousarray(shared_bf16, dtype=np.uint16)
    T, K = perm.shape
    H = rows.shape[1]
    out = np.empty((T, H), dtype=np.uint16)
    lib().or_finalize(_p(rows), _p(w), _p(perm), _p(sh), _p(out), T, K, H)
    return out


def allreduce_ranks(partials) -> np.ndarray:
    """bf16 bits of the rank-order fp32 sum of the ranks' bf16 partials."""
    y = np.ascontiguousarray(np.stack([np.asarray(p, dtype=np.uint16) for p in partials]))
    out = np.empty(y.shape[1:], dtype=np.uint16)
    lib().or_allreduce_ranks(_p(y), _p(out), y.shape[0], ctypes.c_size_t(out.size))
    return out


def allreduce_norm(partials, residual: np.ndarray, gamma: Optional[np.ndarray], eps: float):
    """(residual_out, norm_out) bf16 bits of the all-reduce + residual + RMSNorm
    epilogue over the ranks' bf16 partials (norm_out None without gamma)."""
    y = np.ascontiguousarray(np.stack([np.asarray(p, dtype=np.uint16) for p in partials]))
    world, T, H = y.shape
    res = np.ascontiguousarray(residual, dtype=np.uint16)
    gam = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.uint16)
    r_out = np.empty((T, H), dtype=np.uint16)
    n_out = None if gam is None else np.empty((T, H), dtype=np.uint16)
    lib().or_allreduce_norm(_p(y), _p(res), _p(gam), c_float(eps), _p(r_out), _p(n_out), world, T, H)
    return r_out, n_out


def ref_route_lib() -> Optional[ctypes.CDLL]:
    """The reference's own route kernels compiled for the CPU (oracle/_ref), or None."""
    if not os.path.exists(REF_LIB):
        return None
    return ctypes.CDLL(REF_LIB)


# --------------------------------------------------------------------- codecs / MLP
def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def dequant_mxfp4(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """u8 [..., K/2] codes + u8 [..., K/32] E8M0 -> fp32 [..., K] (exact)."""
    lut = torch.from_numpy(E2M1)
    lo = lut[(codes & 0x0F).long()]
    hi = lut[(codes >> 4).long()]
    vals = torch.stack([lo, hi], dim=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)
    sc = torch.exp2(scales.float() - 127.0)
    return (vals.reshape(*scales.shape, 32) * sc[..., None]).reshape(vals.shape)


def expert_mlp(x: torch.Tensor, w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
               clamp: Optional[float], numerics: str, terms: int = 3, nv: Optional[tuple] = None) -> torch.Tensor:
    """fp32 [n, H] of one expert on fp32 rows x [n, H] (CPU). ``nv`` = (w13
    scale_2, w2 scale_2, (fc1 input scale, fc2 input scale)) for NVFP4 weights."""
    inter = w13.shape[0] // 2
    fmt = "nvfp4" if nv is not None else "mxfp4"
    W13 = dequant_nvfp4(w13, s13, nv[0]) if nv is not None else dequant_mxfp4(w13, s13)
    xin = x
    if numerics == "kernel":
        xin = torch.from_numpy(act_roundtrip(x.numpy(), terms, fmt, nv[2][0] if nv is not None else 1.0))
    gu = xin @ W13.T
    gate, up = gu[:, :inter], gu[:, inter:]
    if clamp is not None:
        up = up.clamp(-clamp, clamp)
        gate = gate.clamp(max=clamp)
    h = up * (gate * torch.sigmoid(gate))
    if numerics == "kernel":
        h = torch.from_numpy(act_roundtrip(h.numpy(), terms, fmt, nv[2][1] if nv is not None else 1.0))
    W2 = dequant_nvfp4(w2, s2, nv[1]) if nv is not None else dequant_mxfp4(w2, s2)
    return h @ W2.T


def moe_layer(x_bf16: torch.Tensor, ids: np.ndarray, weights: np.ndarray, layer: dict, *, numerics: str = "exact",
              terms: int = 3, expert_offset: int = 0, local_experts: Optional[int] = None, deal_group: int = -1):
    """Oracle of one MoE layer given routing. Returns (out fp32 [T, H] before
    bf16 rounding of the final sum, per-slot rows fp32 {(t, k): [H]}, shared
    fp32 [T, H] or None). Weights are CPU uint8 tensors in the canonical layout."""
    x = x_bf16.float()
    T = x.shape[0]
    w13, s13, w2, s2 = layer["w13"], layer["w13_scale"], layer["w2"], layer["w2_scale"]
    E = w13.shape[0] if local_experts is None else local_experts
    clamp = layer.get("clamp")
    rows = {}
    by_expert = {}
    dealt = None
    if deal_group >= 0:  # balanced dealing: the step's distinct experts, k-th to group k % 2
        present = sorted({int(i) for i in ids.flatten() if 0 <= int(i) < E})
        dealt = {e for r, e in enumerate(present) if r % 2 == deal_group}
    for t in range(T):
        for k in range(ids.shape[1]):
            e = int(ids[t, k]) - expert_offset
            if 0 <= e < E and (dealt is None or e in dealt):
                by_expert.setdefault(e, []).append((t, k))
    nvl = layer.get("fmt") == "nvfp4"
    ins = layer.get("input_scale")

    def nv_of(sc13, sc2, e):
        return (float(sc13[e]), float(sc2[e]), ins) if nvl else None

    for e, slots in sorted(by_expert.items()):
        toks = torch.tensor([t for t, _ in slots])
        lim = None if clamp is None else float(clamp[e])
        y = expert_mlp(x[toks], w13[e], s13[e], w2[e], s2[e], lim, numerics, terms,
                       nv_of(layer.get("w13_scale_2"), layer.get("w2_scale_2"), e))
        for j, slot in enumerate(slots):
            rows[slot] = y[j]
    shared = None
    if layer.get("shared") is not None:
        sw = layer["shared"]
        lim = layer.get("shared_clamp")
        shared = expert_mlp(x, sw[0][0], sw[1][0], sw[2][0], sw[3][0], lim, numerics, terms,
                            nv_of(sw[4], sw[5], 0) if nvl else None)
    out = torch.zeros_like(x)
    for (t, k), y in rows.items():
        out[t] += float(weights[t, k]) * y
    if shared is not None:
        out = out + shared
    return out, rows, shared


# --------------------------------------------------------------------- seeded inputs
def make_layer(H: int, I: int, E: int, *, shared: bool, seed: int, scale_lo: int = 117, scale_hi: int = 121,
               clamp: Optional[float] = None, generator_device: str = "cpu") -> dict:
    """Seeded MXFP4 layer (canonical layout): E2M1 codes uniform over the 16
    nibbles, E8M0 bytes uniform in [scale_lo, scale_hi] (exponents -10..-6)."""
    g = torch.Generator(device=generator_device).manual_seed(seed)

    def rnd(shape, lo, hi):
        return torch.randint(lo, hi + 1, shape, dtype=torch.uint8, generator=g, device=generator_device)

    layer = {
        "w13": rnd((E, 2 * I, H // 2), 0, 255),
        "w13_scale": rnd((E, 2 * I, H // 32), scale_lo, scale_hi),
        "w2": rnd((E, H, I // 2), 0, 255),
        "w2_scale": rnd((E, H, I // 32), scale_lo, scale_hi),
        "clamp": None if clamp is None else torch.full((E,), float(clamp)),
        "shared": None,
    }
    if shared:
        layer["shared"] = (rnd((1, 2 * I, H // 2), 0, 255), rnd((1, 2 * I, H // 32), scale_lo, scale_hi),
                           rnd((1, H, I // 2), 0, 255), rnd((1, H, I // 32), scale_lo, scale_hi))
    return layer


def make_nvfp4_layer(H: int, I: int, E: int, *, shared: bool, seed: int, sf_lo: float = 0.5, sf_hi: float = 4.0,
                     clamp: Optional[float] = None) -> dict:
    """Seeded NVFP4 layer (canonical ModelOpt layout): E2M1 codes uniform over
    the 16 nibbles, E4M3 scales of values ~U[sf_lo, sf_hi] per 16 elements, a
    per-expert fp32 scale_2 of 2^-8 (1 + u/4), u ~ U[0, 1); the static input
    scales are calibrated on a sample: FC1 for |x| <= 8, FC2 for twice the
    largest |h| of 8 rows of x ~ N(0, 1) through expert 0."""
    g = torch.Generator().manual_seed(seed)

    def rnd(shape):
        return torch.randint(0, 256, shape, dtype=torch.uint8, generator=g)

    def sf(shape):
        v = sf_lo + (sf_hi - sf_lo) * torch.rand(shape, generator=g)
        return v.to(torch.float8_e4m3fn).view(torch.uint8)

    def s2(n):
        return (2.0 ** -8 * (1.0 + 0.25 * torch.rand((n,), generator=g))).float()

    layer = {
        "fmt": "nvfp4",
        "w13": rnd((E, 2 * I, H // 2)), "w13_scale": sf((E, 2 * I, H // 16)),
        "w2": rnd((E, H, I // 2)), "w2_scale": sf((E, H, I // 16)),
        "w13_scale_2": s2(E), "w2_scale_2": s2(E),
        "clamp": None if clamp is None else torch.full((E,), float(clamp)),
        "shared": None,
    }
    if shared:
        layer["shared"] = (rnd((1, 2 * I, H // 2)), sf((1, 2 * I, H // 16)), rnd((1, H, I // 2)),
                           sf((1, H, I // 16)), s2(1), s2(1))
    fc1 = 8.0 / (6.0 * 448.0)
    xs = torch.randn((8, H), generator=g)
    W13 = dequant_nvfp4(layer["w13"][0], layer["w13_scale"][0], float(layer["w13_scale_2"][0]))
    gu = xs @ W13.T
    h = gu[:, I:] * (gu[:, :I] * torch.sigmoid(gu[:, :I]))
    fc2 = 2.0 * float(h.abs().max()) / (6.0 * 448.0)
    layer["input_scale"] = (float(np.float32(fc1)), float(np.float32(fc2)))
    return layer


def make_inputs(T: int, H: int, E: int, seed: int, router: bool = True):
    """x bf16 ~ N(0, 1) [T, H], router weight bf16 ~ N(0, 0.02) [E, H], bias ~ N(0, 0.01)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    w = (torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16) if router else None
    bias = (torch.randn((E,), generator=g) * 0.01).float()
    return x, w, bias


def max_abs_rel(got: np.ndarray, ref: np.ndarray) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))
