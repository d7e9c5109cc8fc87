"""Host wrappers of the bit-packed CUDA kernels, and parameter -> truth-table conversion.

Packed activations are int64 tensors ``[rows, ldw]`` (conv: ``[C, H, W, ldw]``)
with ``ldw = ceil(B/64)`` rounded up to even; sample ``b`` is bit ``b % 64`` of
word ``b // 64``, as in ``silogic/bitpacking/ops.py:32-49``.
"""
import ctypes
import weakref

import torch

from . import _lib
from ._lib import call, lib, ptr, require_cuda, stream_ptr
from .functional import gate16_lut_codes

_GATE_LUT = gate16_lut_codes()


def n_words(B):
    """Number of 64-sample words for ``B`` samples (``ops.py:27-29``)."""
    return (int(B) + 63) >> 6


def ldw_for(B):
    nw = n_words(B)
    return max(2, nw + (nw & 1))


# ------------------------------------------------------------------ packing
def pack(x, ldw=None):
    """``[B, F]`` (uint8 / bool / float, nonzero-after-uint8-cast = 1) -> ``[F, ldw]`` int64."""
    require_cuda(x)
    B = x.shape[0]
    x2 = x.reshape(B, -1)
    F = x2.shape[1]
    ldw = ldw or ldw_for(B)
    out = torch.empty((F, ldw), dtype=torch.int64, device=x.device)
    if x2.dtype == torch.bool:
        x2 = x2.view(torch.uint8)
    if x2.dtype == torch.uint8:
        x2 = x2.contiguous()
        call("slg_pack_u8", ptr(x2), B, F, ptr(out), ldw, stream_ptr(x.device))
    else:
        x2 = x2.float().contiguous()
        call("slg_pack_f32", ptr(x2), B, F, ptr(out), ldw, stream_ptr(x.device))
    return out


def unpack(p, B):
    """``[F, ldw]`` int64 -> ``[B, F]`` uint8."""
    require_cuda(p)
    p = p.contiguous()
    F, ldw = p.shape[0], p.shape[-1]
    F = p.numel() // ldw
    out = torch.empty((B, F), dtype=torch.uint8, device=p.device)
    call("slg_unpack_u8", ptr(p), F, ldw, B, ptr(out), stream_ptr(p.device))
    return out


_THR_CACHE = {}


def _thresholds(thresholds, device):
    """Shared thresholds as a device tensor (cached for Python sequences) + sortedness."""
    if isinstance(thresholds, (list, tuple)):
        key = (tuple(float(t) for t in thresholds), str(device))
        hit = _THR_CACHE.get(key)
        if hit is None:
            vals = [float(t) for t in thresholds]
            t = torch.tensor(vals, dtype=torch.float32).to(device)
            hit = (t, all(a <= b for a, b in zip(vals, vals[1:])))
            _THR_CACHE[key] = hit
        return hit
    t = torch.as_tensor(thresholds, dtype=torch.float32, device=device).contiguous()
    return t, False


def thermo_pack(img, thresholds, mode=0, ldw=None):
    """Thermometer-encode ``[B, C, H, W]`` fp32 -- or uint8, pixel k read as the fp32
    quotient k / 255 as torchvision's ``ToTensor`` gives it -- and pack to
    ``[C*T, H, W, ldw]``.

    mode 0 = ``binarize_spatial`` (shared thresholds, channel ``t*C + c``; a sorted
    Python sequence takes the binary-search kernel path);
    mode 1 = learned encoder (per-feature thresholds ``[C*H*W, T]``, channel ``c*T + t``).
    """
    require_cuda(img)
    B, C, H, W = img.shape
    if mode == 0:
        thr, is_sorted = _thresholds(thresholds, img.device)
        if is_sorted:
            mode = 2
    else:
        thr = torch.as_tensor(thresholds, dtype=torch.float32, device=img.device).contiguous()
    T = thr.shape[-1] if thr.dim() else 1
    ldw = ldw or ldw_for(B)
    out = torch.empty((C * T, H, W, ldw), dtype=torch.int64, device=img.device)
    mode = int(mode)
    if img.dtype == torch.uint8:    # pixel k read as k / 255 (ToTensor), a quarter of the bytes
        x = img.contiguous()
        call("slg_thermo_pack_u8", ptr(x), B, C, H * W, ptr(thr), T, mode, ptr(out), ldw,
             stream_ptr(img.device))
    else:
        x = img.float().contiguous()
        call("slg_thermo_pack", ptr(x), B, C, H * W, ptr(thr), T, mode, ptr(out), ldw,
             stream_ptr(img.device))
    return out


# ----------------------------------------------------------- wiring checks
_CHECKED = {}   # id(index tensor) -> (weakref to it, version, limit) that passed


def check_index_range(idx, limit, what="index"):
    """Raise ``IndexError`` unless every entry of ``idx`` lies in ``[0, limit)``.

    The kernels trust their wiring (an index out of range is an out-of-bounds device
    read), so every circuit is checked once when it is built or loaded: FC wiring
    against the layer's input width, conv leaves against ``cin * k * k``, soft
    candidates against the input width.  CUDA tensors go through the library's
    ``slg_check_index_range`` (one small kernel + a synchronisation); host tensors are
    checked on the host.  A tensor that passed is remembered until it is modified
    in place (its version counter changes).
    """
    if idx is None or idx.numel() == 0:
        return
    if torch.compiler.is_compiling():      # host validation; the eager call checked it
        return
    seen = _CHECKED.get(id(idx))
    if seen is not None and seen[0]() is idx and seen[1] == idx._version and seen[2] <= limit:
        return
    if idx.is_cuda:
        i32 = idx if idx.dtype == torch.int32 else idx.to(torch.int32)
        if idx.dtype != torch.int32 and (idx.min() < -2**31 or idx.max() >= 2**31):
            raise IndexError(f"{what}: entries do not fit in int32")
        i32 = i32.contiguous()
        scratch = torch.empty(2, dtype=torch.int64, device=idx.device)
        st = lib().slg_check_index_range(ptr(i32), i32.numel(), int(limit), ptr(scratch),
                                         stream_ptr(idx.device))
        if st != 0:
            raise IndexError(f"{what}: " + lib().slg_last_error().decode(errors="replace"))
    else:
        lo, hi = int(idx.min()), int(idx.max())
        if lo < 0 or hi >= limit:
            raise IndexError(f"{what}: index out of range: entries span [{lo}, {hi}], "
                             f"allowed [0, {limit})")
    if len(_CHECKED) > 4096:
        for k in [k for k, v in _CHECKED.items() if v[0]() is None]:
            del _CHECKED[k]
    _CHECKED[id(idx)] = (weakref.ref(idx), idx._version, int(limit))


# ---------------------------------------------------------------- circuits
def fc(x, idx, tt, wire_r=0, out=None):
    """One FC hard layer: ``[in, ldw]`` -> ``[out, ldw]``."""
    require_cuda(x)
    in_dim, ldw = x.shape
    out_dim, arity = idx.shape
    if out is None:
        out = torch.empty((out_dim, ldw), dtype=torch.int64, device=x.device)
    call("slg_fc_hard", ptr(x), in_dim, ldw, ptr(idx), ptr(tt), arity, out_dim, wire_r,
         ptr(out), stream_ptr(x.device))
    return out


def conv(x, leaf, tt, arity, depth, kernel=3, pad=1, wire_r=0, pool=2, out=None):
    """One conv tree block (+ OR-pool): ``[C, H, W, ldw]`` -> ``[n, Ho/pool, Wo/pool, ldw]``."""
    require_cuda(x)
    C, H, W, ldw = x.shape
    n = leaf.shape[0]
    Ho, Wo = H + 2 * pad - kernel + 1, W + 2 * pad - kernel + 1
    if out is None:
        out = torch.empty((n, Ho // pool, Wo // pool, ldw), dtype=torch.int64, device=x.device)
    call("slg_conv_hard", ptr(x), C, H, W, ldw, ptr(leaf), ptr(tt), arity, depth, kernel, pad,
         n, wire_r, pool, ptr(out), stream_ptr(x.device))
    return out


def groupsum(x, B, num_classes, out=None):
    """Per-sample, per-class popcounts ``[B, C]`` int32 of ``[width, ldw]`` packed rows."""
    require_cuda(x)
    width = x.numel() // x.shape[-1]
    if out is None:
        out = torch.empty((B, num_classes), dtype=torch.int32, device=x.device)
    call("slg_groupsum", ptr(x), width, x.shape[-1], B, num_classes, ptr(out),
         stream_ptr(x.device))
    return out


def packed_linear(x, W, bias, B):
    """Learned readout ``[B, C]`` fp32 = bits of packed ``x`` ``[width, ldw]`` @ ``W.T`` + bias."""
    require_cuda(x)
    W = W.float().contiguous()
    bias = bias.float().contiguous() if bias is not None else None
    width = x.numel() // x.shape[-1]
    out = torch.empty((B, W.shape[0]), dtype=torch.float32, device=x.device)
    call("slg_packed_linear", ptr(x), width, x.shape[-1], B, ptr(W), ptr(bias), W.shape[0], ptr(out),
         stream_ptr(x.device))
    return out


# ------------------------------------------- whole FC stack in one launch
CHAIN_MAX_LAYERS = 32
CHAIN_MAX_WIDTH = 13824
CHAIN_MAX_CLASSES = 64
CHAIN_MAX_SMEM = 227 * 1024           # opt-in shared memory per CTA on sm_100


def chain_encode(idx, tt, wire_r=0):
    """One arity-2 layer's wiring ``[out, 2]`` + tables ``[out]`` -> ``[out]`` int32 records."""
    require_cuda(tt)
    out_dim = tt.shape[0]
    rec = torch.empty(out_dim, dtype=torch.int32, device=tt.device)
    call("slg_fc_chain_encode", ptr(idx.contiguous()), ptr(tt.contiguous()), out_dim, wire_r,
         ptr(rec), stream_ptr(tt.device))
    return rec


def chain_layout(steps, in_dim, num_classes, reorder=True):
    """Node records, layer widths and class offsets for :class:`FCChain`, planned by the
    library's host-side planner ``slg_fc_chain_plan`` (bank-conflict-free half-warps,
    padded layers, per-class blocks in the last layer).  Returns ``(records uint32
    numpy, widths, class offsets)``; record = in_a | in_b << 14 | table << 28 over
    storage slots."""
    import numpy as np
    outs = np.array([st["idx"].shape[0] for st in steps], dtype=np.int64)
    idx = np.ascontiguousarray(np.concatenate(
        [st["idx"].detach().cpu().numpy().astype(np.int32).reshape(-1) for st in steps]))
    tt = np.ascontiguousarray(np.concatenate(
        [st["tt"].detach().cpu().numpy().astype(np.int64).view(np.uint64) for st in steps]))
    wr = np.array([int(st["wire_r"]) for st in steps], dtype=np.int64)
    cap = len(steps) * CHAIN_MAX_WIDTH
    rec = np.zeros(cap, dtype=np.uint32)
    widths = np.zeros(len(steps), dtype=np.int32)
    off = np.zeros(num_classes + 1, dtype=np.int32)
    P = ctypes.c_void_p
    call("slg_fc_chain_plan", int(in_dim), len(steps), P(outs.ctypes.data), P(idx.ctypes.data),
         P(tt.ctypes.data), P(wr.ctypes.data), int(num_classes), int(bool(reorder)),
         P(rec.ctypes.data), cap, P(widths.ctypes.data), P(off.ctypes.data))
    return rec[:int(widths.sum())].copy(), widths.tolist(), off.tolist()


class FCChain:
    """Arity-2 FC layers + GroupSum as one persistent kernel (``slg_fc_chain_counts``)."""

    def __init__(self, steps, in_dim, num_classes, device, reorder=True):
        rec, self.widths, self.class_off = chain_layout(steps, in_dim, num_classes, reorder)
        self.rec = torch.from_numpy(rec.view("int32")).to(device)
        self.in_dim, self.num_classes = int(in_dim), int(num_classes)
        self._w = (ctypes.c_int32 * len(self.widths))(*self.widths)
        self._off = (ctypes.c_int32 * len(self.class_off))(*self.class_off)
        # one CTA per SM holds two layers of the column in shared memory
        self.smem_bytes = 2 * max([self.in_dim] + self.widths) * 8
        self.fits = self.smem_bytes <= CHAIN_MAX_SMEM

    @staticmethod
    def supported(steps, in_dim, num_classes):
        if (not steps or len(steps) > CHAIN_MAX_LAYERS or not num_classes
                or num_classes > CHAIN_MAX_CLASSES or in_dim > CHAIN_MAX_WIDTH):
            return False
        for st in steps:
            if st["op"] != "fc" or st["idx"].shape[1] != 2 or st["idx"].shape[0] > CHAIN_MAX_WIDTH:
                return False
        return steps[-1]["idx"].shape[0] % num_classes == 0

    def counts(self, h, B, out=None):
        require_cuda(h)
        if out is None:
            out = torch.empty((B, self.num_classes), dtype=torch.int32, device=h.device)
        call("slg_fc_chain_counts", ptr(h), self.in_dim, h.shape[-1], B, ptr(self.rec),
             ctypes.cast(self._w, ctypes.c_void_p), len(self.widths), self.num_classes,
             ctypes.cast(self._off, ctypes.c_void_p), ptr(out), stream_ptr(h.device))
        return out


# ------------------------------------------------- parameters -> truth tables
def _pack_tt(bits):
    """``[..., P]`` bool -> ``[...]`` int64 with bit p set where ``bits[..., p]``."""
    P = bits.shape[-1]
    w = torch.ones(P, dtype=torch.int64, device=bits.device) << torch.arange(P, device=bits.device)
    return (bits.to(torch.int64) * w).sum(-1)


def _corners(n, device):
    p = torch.arange(2 ** n, device=device).unsqueeze(1)
    return (p >> torch.arange(n, device=device)) & 1        # [P, n]


@torch.no_grad()
def node_truth_tables(node, params, arity, mono_mask=None):
    """Hard truth tables (int64, bit p = output at address sum_j in_j << j).

    Mirrors each node's ``forward_hard`` evaluated at the 2^arity cube corners
    (``silogic/nodes.py:101-106,153-156,184-189,232-233,266-268``; the corner
    enumeration of ``bitpacking/convert.py:100-123``).
    """
    dev = params.device
    if node == "gate16":
        return _GATE_LUT.to(dev)[params.argmax(dim=-1)]
    if node in ("multilinear", "hybrid"):
        return _pack_tt(params > 0)
    cb = _corners(arity, dev).to(torch.float32)              # [P, n]
    P = 2 ** arity
    if node == "walsh":
        u = 2 * cb - 1
        z = torch.zeros(params.shape[:-1] + (P,), dtype=torch.float32, device=dev)
        for m in range(P):                                   # sum over monomials in order
            mono = torch.ones(P, device=dev)
            for j in range(arity):
                if (m >> j) & 1:
                    mono = mono * u[:, j]
            z = z + params[..., m:m + 1].float() * mono
        return _pack_tt(z > 0)
    if node == "linear":
        z = params[..., :1].float() + params[..., 1:].float() @ cb.t()
        return _pack_tt(z >= 0)
    if node == "polynomial":
        mk = mono_mask.to(dev).float()                       # [M, n]
        mono = torch.where(mk[None] > 0, cb[:, None, :], torch.ones_like(cb[:, None, :])).prod(-1)
        return _pack_tt(params.float() @ mono.t() >= 0)
    raise ValueError(f"no hard form for node {node!r}")
