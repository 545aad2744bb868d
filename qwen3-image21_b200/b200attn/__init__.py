"""Python binding of libb200attn.so (the C ABI in include/b200_attn.h) for tests and
benchmarks.  Every compute call goes through the CUDA library; there is no fallback —
without the built library on an sm_100 device the calls raise.

Names mirror the reference's functions on this path:
  chunked_attention      src/transformer.rs:259  (q, k, v [B,H,S,D], scale, mask)
  flash_attention        src/transformer.rs:243-254 (q, k, v [B,S,H,D], scale; the FA2
                         branch, candle_flash_attn::flash_attn with causal = false)
  attention_forward      src/transformer.rs:179-193 (the norm -> RoPE -> cat -> attention
                         -> head-merge span of Attention::forward)
  joint_layout           src/joint_layout.rs:52  (JointLayout::new)
  rope_positions/rope_pe src/rope.rs:104-211     (EmbedNd)
  key_valid_to_desc      src/transformer.rs:642-649, 736-745
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200attn.so")
HEAD_DIM = 128

# b200_status
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE, ERR_LAYOUT, ERR_DEVICE_TIMEOUT = (
    0, -1, -2, -3, -4, -5, -6)

EXPORTED = (
    "b200_attn_workspace_bytes", "b200_attn_fwd", "b200_joint_attention", "b200_chunked_attention",
    "b200_flash_attention", "b200_flash_attention_ex",
    "b200_norm_rope", "b200_qk_norm_rope",
    "b200_joint_layout", "b200_rope_positions", "b200_rope_pe", "b200_key_valid_to_desc",
    "b200_block_causal_limits",
    "b200_strerror", "b200_attn_strerror", "b200_abi_version",
    "b200_residual_adaln", "b200_swiglu",
    "b200_dequant_q4_k", "b200_dequant_q6_k", "b200_wait_selftest", "b200_gemm",
    "b200_gemm_scatter", "b200_reduce_gather_bf16", "b200_reduce_residual_adaln_gather",
    "b200_reduce_nvls", "b200_kquant_gemv",
    "b200_qkv_norm_rope_gemm",
    "b200_tp_unique_id", "b200_tp_init", "b200_tp_init_from_nccl", "b200_tp_rank", "b200_tp_size",
    "b200_tp_out_proj_allreduce", "b200_tp_wait", "b200_tp_destroy",
)


class B200Error(RuntimeError):
    """A non-zero b200_status from the library."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {strerror(status)} ({status})")


class KvDesc(ctypes.Structure):
    _fields_ = [("prefix_valid", ctypes.c_int32), ("target_valid", ctypes.c_int32)]


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("target_len", ctypes.c_int32), ("prefix_len", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("prefix_k", ctypes.c_void_p), ("prefix_v", ctypes.c_void_p),
        ("norm_q_w", ctypes.c_void_p), ("norm_k_w", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float), ("pe", ctypes.c_void_p), ("desc", ctypes.c_void_p),
        ("scale", ctypes.c_float), ("out", ctypes.c_void_p), ("k_rot_out", ctypes.c_void_p),
        ("v_out", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t), ("status", ctypes.c_void_p),
        ("row_limit", ctypes.c_void_p), ("pe_batch_stride", ctypes.c_int64),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded C-ABI library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with qwen3-image21_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_float
        L.b200_attn_workspace_bytes.argtypes = [ctypes.POINTER(AttnArgs), ctypes.POINTER(ctypes.c_size_t)]
        L.b200_attn_fwd.argtypes = [ctypes.POINTER(AttnArgs), vp]
        L.b200_chunked_attention.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, vp, vp, vp]
        L.b200_flash_attention.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, vp, vp, vp]
        L.b200_flash_attention_ex.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, vp, i32,
                                              vp, vp]
        L.b200_norm_rope.argtypes = [vp, vp, i32, i32, i32, i32, vp, f32, vp, vp]
        L.b200_qk_norm_rope.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, vp, vp, f32, vp, vp]
        L.b200_joint_attention.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, f32, vp,
                                           vp, ctypes.c_size_t, vp, vp]
        L.b200_joint_layout.argtypes = [i32, vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]
        L.b200_rope_positions.argtypes = [vp, i32, vp, i32, vp]
        L.b200_rope_pe.argtypes = [vp, i32, vp, i32, vp, f32, vp]
        L.b200_key_valid_to_desc.argtypes = [vp, i32, i32, i32, vp]
        L.b200_block_causal_limits.argtypes = [vp, i32, vp]
        i64 = ctypes.c_int64
        L.b200_residual_adaln.argtypes = [vp, vp, vp, vp, vp, i64, i32, i64, i64, f32, vp]
        L.b200_swiglu.argtypes = [vp, vp, i64, i32, vp]
        L.b200_dequant_q4_k.argtypes = [vp, vp, i64, vp]
        L.b200_dequant_q6_k.argtypes = [vp, vp, i64, vp]
        L.b200_wait_selftest.argtypes = [vp, ctypes.c_uint32, vp]
        L.b200_gemm.argtypes = [vp, i64, vp, i64, vp, i64, i32, i32, i32, i32, vp, vp]
        L.b200_gemm_scatter.argtypes = [vp, i64, vp, i64, vp, i32, i32, i32, i64, i32, i32, i32, vp, vp]
        L.b200_reduce_gather_bf16.argtypes = [vp, i32, i32, i32, i32, i64, vp, i32, i64, i64, vp]
        L.b200_reduce_residual_adaln_gather.argtypes = [vp, i32, i32, i32, i32, i64, vp, i64, vp, vp,
                                                        i64, i64, f32, vp, i32, i64, i64, vp]
        L.b200_reduce_nvls.argtypes = [vp, i64, vp, i64, i64, i32, i32, vp, i64, vp, vp, i64, i64,
                                       f32, vp]
        L.b200_kquant_gemv.argtypes = [vp, i64, vp, i32, vp, i64, i32, i32, i32, vp]
        L.b200_tp_unique_id.argtypes = [vp]
        L.b200_tp_init.argtypes = [ctypes.POINTER(vp), vp, i32, i32, ctypes.c_uint32]
        L.b200_tp_init_from_nccl.argtypes = [ctypes.POINTER(vp), vp, ctypes.c_uint32]
        L.b200_tp_rank.argtypes = [vp]
        L.b200_tp_size.argtypes = [vp]
        L.b200_tp_out_proj_allreduce.argtypes = [vp, vp, ctypes.c_size_t, i32, vp]
        L.b200_tp_wait.argtypes = [vp, vp]
        L.b200_tp_destroy.argtypes = [vp]
        L.b200_qkv_norm_rope_gemm.argtypes = [vp, i64, vp, i32, i32, i32, i32, vp, vp, f32, vp, i64,
                                              vp, vp, vp, vp, vp]
        L.b200_strerror.argtypes = [ctypes.c_int]
        L.b200_strerror.restype = ctypes.c_char_p
        L.b200_attn_strerror.restype = ctypes.c_char_p
        for name in EXPORTED:
            if name != "b200_strerror":
                getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def strerror(status: int) -> str:
    return lib().b200_strerror(int(status)).decode()


def _check(rc: int, what: str) -> None:
    if rc != OK:
        raise B200Error(rc, what)


def _np_ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------- host-side mirrors
def joint_layout(text_len: int, text_image_mask: Optional[Sequence[bool]],
                 cond_shapes: Sequence[Tuple[int, int]], target: Tuple[int, int]) -> dict:
    """JointLayout::new via the C ABI: image_ids, image_pad_mask, img_shapes, lengths."""
    tim = None if text_image_mask is None else np.ascontiguousarray(text_image_mask, np.uint8)
    cs = np.ascontiguousarray(np.asarray(cond_shapes, np.int32).reshape(-1, 2)) if len(cond_shapes) else None
    n_cond = 0 if cs is None else cs.shape[0]
    ln, pl, tl = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    shapes = np.zeros((n_cond + 1, 3), np.int32)
    _check(lib().b200_joint_layout(text_len, _np_ptr(tim), _np_ptr(cs), n_cond, target[0], target[1],
                                   0, None, None, _np_ptr(shapes), ctypes.byref(ln),
                                   ctypes.byref(pl), ctypes.byref(tl)), "joint_layout")
    ids = np.zeros(ln.value, np.int64)
    mask = np.zeros(ln.value, np.uint8)
    _check(lib().b200_joint_layout(text_len, _np_ptr(tim), _np_ptr(cs), n_cond, target[0], target[1],
                                   ln.value, _np_ptr(ids), _np_ptr(mask), _np_ptr(shapes),
                                   ctypes.byref(ln), ctypes.byref(pl), ctypes.byref(tl)), "joint_layout")
    return dict(image_ids=ids, image_pad_mask=mask, img_shapes=[tuple(map(int, s)) for s in shapes],
                prefix_len=pl.value, target_len=tl.value)


def rope_positions(img_shapes, image_pad_mask) -> np.ndarray:
    """EmbedNd position rules via the C ABI -> int64 [S, 3]."""
    shp = np.ascontiguousarray(np.asarray(img_shapes, np.int32).reshape(-1, 3))
    m = np.ascontiguousarray(image_pad_mask, np.uint8)
    out = np.zeros((m.shape[0], 3), np.int64)
    _check(lib().b200_rope_positions(_np_ptr(shp), shp.shape[0], _np_ptr(m), m.shape[0], _np_ptr(out)),
           "rope_positions")
    return out


def rope_pe(img_shapes, image_pad_mask, axes=(16, 56, 56), theta: float = 1e4) -> np.ndarray:
    """EmbedNd::new + forward via the C ABI -> float32 [S, sum(axes)]."""
    shp = np.ascontiguousarray(np.asarray(img_shapes, np.int32).reshape(-1, 3))
    m = np.ascontiguousarray(image_pad_mask, np.uint8)
    ax = np.ascontiguousarray(axes, np.int32)
    out = np.zeros((m.shape[0], int(sum(axes))), np.float32)
    _check(lib().b200_rope_pe(_np_ptr(shp), shp.shape[0], _np_ptr(m), m.shape[0], _np_ptr(ax),
                              float(theta), _np_ptr(out)), "rope_pe")
    return out


def block_causal_limits(image_ids) -> np.ndarray:
    """Per-row key limits of the block-causal mask (src/attention_mask.rs:18-66)."""
    ids = np.ascontiguousarray(image_ids, np.int64)
    out = np.zeros(ids.shape[0], np.int32)
    _check(lib().b200_block_causal_limits(_np_ptr(ids), ids.shape[0], _np_ptr(out)),
           "block_causal_limits")
    return out


def key_valid_to_desc(key_valid: np.ndarray, prefix_len: int, target_len: int) -> np.ndarray:
    """[B, P+T] 0/1 mask -> int32 [B, 2] descriptors (prefix_valid, target_valid)."""
    kv = np.ascontiguousarray(key_valid, np.uint8)
    out = np.zeros((kv.shape[0], 2), np.int32)
    _check(lib().b200_key_valid_to_desc(_np_ptr(kv), kv.shape[0], prefix_len, target_len, _np_ptr(out)),
           "key_valid_to_desc")
    return out


# ----------------------------------------------------------------- device entry points
def _stream(stream) -> Optional[int]:
    import torch
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _dptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def make_args(q, k, v, prefix_k, prefix_v, norm_q_w, norm_k_w, pe, out, desc=None, scale=None,
              eps: float = 1e-6, k_rot_out=None, v_out=None, workspace=None, status=None,
              row_limit=None) -> AttnArgs:
    """Fill b200_attn_args from torch tensors (no checks beyond what the library does)."""
    b, t, h, d = q.shape
    p = 0 if prefix_k is None else prefix_k.shape[2]
    a = AttnArgs()
    a.batch, a.heads, a.head_dim, a.target_len, a.prefix_len = b, h, d, t, p
    a.q, a.k, a.v = _dptr(q), _dptr(k), _dptr(v)
    a.prefix_k, a.prefix_v = _dptr(prefix_k), _dptr(prefix_v)
    a.norm_q_w, a.norm_k_w = _dptr(norm_q_w), _dptr(norm_k_w)
    a.norm_eps = eps
    a.pe = _dptr(pe)
    # pe [T, D] is shared by the batch rows; pe [B, T, D] gives each row its own table.
    a.pe_batch_stride = pe.shape[-2] * pe.shape[-1] if pe is not None and pe.dim() == 3 else 0
    a.desc = _dptr(desc)
    a.scale = d ** -0.5 if scale is None else scale
    a.out = _dptr(out)
    a.k_rot_out, a.v_out = _dptr(k_rot_out), _dptr(v_out)
    a.workspace = _dptr(workspace)
    a.workspace_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    a.status = _dptr(status)
    a.row_limit = _dptr(row_limit)
    return a


def workspace_bytes(args: AttnArgs) -> int:
    n = ctypes.c_size_t()
    _check(lib().b200_attn_workspace_bytes(ctypes.byref(args), ctypes.byref(n)), "workspace_bytes")
    return n.value


def attention_forward(q, k, v, prefix_k, prefix_v, norm_q_w, norm_k_w, pe, desc=None, scale=None,
                      eps: float = 1e-6, out=None, k_rot_out=None, v_out=None, workspace=None,
                      status=None, stream=None, row_limit=None):
    """The Attention::forward span from the norm to the head merge on the GPU.

    q, k, v: bf16 [B,T,H,D] raw projections; prefix_k/v: bf16 [B,H,P,D] (or None);
    norm weights f32 [D]; pe f32 [T,D] (or [B,T,D], one table per batch row); desc int32
    [B,2] device tensor or None.
    Returns out bf16 [B,T,H*D].
    """
    import torch
    b, t, h, d = q.shape
    if out is None:
        out = torch.empty((b, t, h * d), dtype=torch.bfloat16, device=q.device)
    args = make_args(q, k, v, prefix_k, prefix_v, norm_q_w, norm_k_w, pe, out, desc, scale, eps,
                     k_rot_out, v_out, None, status, row_limit)
    if workspace is None:
        need = workspace_bytes(args)
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel()
    _check(lib().b200_attn_fwd(ctypes.byref(args), _stream(stream)), "b200_attn_fwd")
    return out


def flash_attention(q, k, v, scale: float, key_len=None, status=None, out=None, stream=None):
    """flash_attention / flash_attn(q, k, v, scale, causal=False) on [B,S,H,D] tensors
    (token-major, no transposes) -> out [B,Sq,H,D] of the same type.  bf16 or float16 (the
    type the reference's FA2 branch casts to); any other dtype raises B200Error
    ERR_UNSUPPORTED from the library.  ``key_len`` (int32 device tensor [B]): batch row b
    attends to keys [0, key_len[b])."""
    import torch
    b, sq, h, d = q.shape
    skv = k.shape[1]
    dtype = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}.get(q.dtype, -1)
    if out is None:
        out = torch.empty((b, sq, h, d), dtype=q.dtype, device=q.device)
    _check(lib().b200_flash_attention_ex(_dptr(q), _dptr(k), _dptr(v), _dptr(out), b, sq, skv, h,
                                         d, float(scale), _dptr(key_len), dtype, _dptr(status),
                                         _stream(stream)),
           "b200_flash_attention_ex")
    return out


def chunked_attention(q, k, v, scale: float, mask=None, key_len=None, status=None, out=None,
                      stream=None):
    """chunked_attention(q, k, v, scale, mask) on [B,H,S,D] bf16 tensors.

    ``mask`` is the reference's bool key mask [B,1,1,Skv] (True = attend); it must keep a
    leading run of keys per batch row (B200Error ERR_LAYOUT otherwise).  ``key_len`` (int32
    device tensor [B]) may be given instead.
    """
    import torch
    b, h, sq, d = q.shape
    skv = k.shape[2]
    if mask is not None:
        if key_len is not None:
            raise ValueError("give mask or key_len, not both")
        m = mask.reshape(b, -1)
        if m.shape[1] != skv:
            raise B200Error(ERR_LAYOUT, "chunked_attention: per-query masks are not supported")
        m = m.to("cpu").numpy().astype(bool)
        lens = m.sum(1)
        for i in range(b):
            if not m[i, :lens[i]].all():
                raise B200Error(ERR_LAYOUT, "chunked_attention: mask is not a leading run of keys")
        key_len = torch.tensor(lens, dtype=torch.int32, device=q.device)
    if out is None:
        out = torch.empty((b, h, sq, d), dtype=torch.bfloat16, device=q.device)
    _check(lib().b200_chunked_attention(_dptr(q), _dptr(k), _dptr(v), _dptr(out), b, h, sq, skv, d,
                                        float(scale), _dptr(key_len), _dptr(status), _stream(stream)),
           "b200_chunked_attention")
    return out


def norm_rope(x, norm_w, eps: float, pe, out=None, stream=None):
    """RMSNorm + RoPE: x bf16 [B,T,H,D] -> bf16 [B,H,T,D]."""
    import torch
    b, t, h, d = x.shape
    if out is None:
        out = torch.empty((b, h, t, d), dtype=torch.bfloat16, device=x.device)
    _check(lib().b200_norm_rope(_dptr(x), _dptr(out), b, t, h, d, _dptr(norm_w), float(eps), _dptr(pe),
                                _stream(stream)), "b200_norm_rope")
    return out


def qk_norm_rope(q, k, norm_q_w, norm_k_w, eps: float, pe, q_rot=None, k_rot=None, stream=None):
    """The b200_attn_fwd prologue alone: RMSNorm + RoPE of q and k in one launch.
    q, k bf16 [B,T,H,D] -> (q_rot, k_rot) bf16 [B,H,T,D]."""
    import torch
    b, t, h, d = q.shape
    if q_rot is None:
        q_rot = torch.empty((b, h, t, d), dtype=torch.bfloat16, device=q.device)
    if k_rot is None:
        k_rot = torch.empty((b, h, t, d), dtype=torch.bfloat16, device=q.device)
    _check(lib().b200_qk_norm_rope(_dptr(q), _dptr(k), _dptr(q_rot), _dptr(k_rot), b, t, h, d,
                                   _dptr(norm_q_w), _dptr(norm_k_w), float(eps), _dptr(pe),
                                   _stream(stream)), "b200_qk_norm_rope")
    return q_rot, k_rot


SPLIT_WORKSPACE_BYTES = 21299968  # B200_ATTN_SPLIT_WORKSPACE_BYTES


def joint_attention(q_rot, k_rot, v, prefix_k, prefix_v, desc=None, scale=None, out=None,
                    workspace=None, status=None, stream=None):
    """The attention launch of b200_attn_fwd: post-RoPE q_rot/k_rot bf16 [B,H,T,D], v bf16
    [B,T,H,D], prefix bf16 [B,H,P,D] or None -> out bf16 [B,T,H*D].  A uint8 device
    ``workspace`` of SPLIT_WORKSPACE_BYTES enables the tail split (None: no split)."""
    import torch
    b, h, t, d = q_rot.shape
    p = 0 if prefix_k is None else prefix_k.shape[2]
    if out is None:
        out = torch.empty((b, t, h * d), dtype=torch.bfloat16, device=q_rot.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().b200_joint_attention(_dptr(q_rot), _dptr(k_rot), _dptr(v), _dptr(prefix_k),
                                      _dptr(prefix_v), b, h, t, p, d, _dptr(desc),
                                      float(d ** -0.5 if scale is None else scale), _dptr(out),
                                      _dptr(workspace), ws_bytes, _dptr(status), _stream(stream)),
           "b200_joint_attention")
    return out


# ----------------------------------------------------------------- block elementwise steps
def residual_adaln(x, y, gate, scale, out, rows_per_mod: int, eps: float = 1e-6, stream=None):
    """x += tanh(gate) * y (if y is given); out = LayerNorm(x) * (1 + scale) (if out is given).

    x f32 [R, C] (updated in place); y bf16 [R, C] or None; gate / scale f32 rows of one
    modulation matrix [n_mod, ...] (row stride taken from the tensor) selected by
    r // rows_per_mod; out bf16 [R, C] or None.  (src/transformer.rs:407-424, 448-454)
    """
    cols = x.shape[-1]
    rows = x.numel() // cols
    strides = {t.stride(0) if t.dim() > 1 else 0 for t in (gate, scale) if t is not None}
    if len(strides) > 1 and rows > rows_per_mod:
        raise ValueError("gate and scale must be rows of one modulation matrix")
    stride = max(strides) if rows > rows_per_mod else 0
    _check(lib().b200_residual_adaln(_dptr(x), _dptr(y), _dptr(gate), _dptr(scale), _dptr(out),
                                     rows, cols, int(rows_per_mod), stride, float(eps),
                                     _stream(stream)), "b200_residual_adaln")
    return out


def swiglu(gp, h=None, stream=None):
    """h = silu(gp[:, :F]) * gp[:, F:] for gp bf16 [R, 2F] (src/transformer.rs:326-331)."""
    import torch
    rows, f2 = gp.numel() // gp.shape[-1], gp.shape[-1]
    if h is None:
        h = torch.empty((rows, f2 // 2), dtype=torch.bfloat16, device=gp.device)
    _check(lib().b200_swiglu(_dptr(gp), _dptr(h), rows, f2 // 2, _stream(stream)), "b200_swiglu")
    return h


# ----------------------------------------------------------------- GGUF k-quant weights
Q4_K_BLOCK_BYTES, Q6_K_BLOCK_BYTES, QK_K = 144, 210, 256


def dequant(blocks, qtype: str, out=None, stream=None):
    """GGUF k-quant super-blocks (uint8 [..., n_blocks * block_bytes]) -> bf16 [n_blocks * 256]
    (viewed as the caller's shape when `out` is given).  qtype: "q4_k" or "q6_k"."""
    import torch
    nbytes = {"q4_k": Q4_K_BLOCK_BYTES, "q6_k": Q6_K_BLOCK_BYTES}[qtype]
    n_blocks = blocks.numel() // nbytes
    if out is None:
        out = torch.empty(n_blocks * QK_K, dtype=torch.bfloat16, device=blocks.device)
    fn = lib().b200_dequant_q4_k if qtype == "q4_k" else lib().b200_dequant_q6_k
    _check(fn(_dptr(blocks), _dptr(out), n_blocks, _stream(stream)), f"b200_dequant_{qtype}")
    return out


def wait_selftest(limit_us: int = 20000, stream=None):
    """Runs the device-side bounded-wait self-test; returns the two status words
    (1, 1 when a wait ran out and the abort flag released the other waiter)."""
    import torch
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    _check(lib().b200_wait_selftest(_dptr(status), int(limit_us), _stream(stream)),
           "b200_wait_selftest")
    return [int(x) for x in status.cpu()]


# ----------------------------------------------------------------- GEMM (tcgen05)
GEMM_STORE_BF16, GEMM_RED_F32 = 0, 1


def gemm(a, b, out=None, mode: int = GEMM_STORE_BF16, c_ptr: Optional[int] = None,
         ldc: Optional[int] = None, status=None, stream=None):
    """a [M, K] bf16 (row stride a.stride(0)) times b [N, K] bf16 (row stride b.stride(0))
    transposed.  mode GEMM_STORE_BF16: out bf16 [M, N] = a @ b.T; GEMM_RED_F32: out f32
    [M, N] += a @ b.T (c_ptr: a raw device address instead, e.g. a peer's buffer)."""
    import torch
    m, k = a.shape
    n = b.shape[0]
    if out is None and c_ptr is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    cp = c_ptr if c_ptr is not None else out.data_ptr()
    if ldc is None:
        ldc = out.stride(0)
    _check(lib().b200_gemm(_dptr(a), a.stride(0), _dptr(b), b.stride(0), cp, ldc, m, n, k, mode,
                           _dptr(status), _stream(stream)), "b200_gemm")
    return out


def _ptr_array(ptrs):
    arr = (ctypes.c_void_p * len(ptrs))(*[int(p) for p in ptrs])
    return arr


def gemm_scatter(a, b, owner_ptrs, src_slot: int, rows_per_owner: int, ldc: int, status=None,
                 stream=None):
    """b200_gemm_scatter: rows of a @ b.T (bf16) into their owners' slots (see the header)."""
    m, k = a.shape
    n = b.shape[0]
    arr = _ptr_array(owner_ptrs)
    _check(lib().b200_gemm_scatter(_dptr(a), a.stride(0), _dptr(b), b.stride(0), arr, len(owner_ptrs),
                                   src_slot, rows_per_owner, ldc, m, n, k, _dptr(status),
                                   _stream(stream)), "b200_gemm_scatter")


def reduce_gather(slots, n_src: int, slot_rows: int, rows: int, cols: int, ld: int, dst_ptrs,
                  dst_row0: int, dst_ld: int, stream=None):
    """b200_reduce_gather_bf16: sum the first `rows` rows of n_src slots (slot_rows rows
    apart) and broadcast them to dst_ptrs at row dst_row0."""
    arr = _ptr_array(dst_ptrs)
    _check(lib().b200_reduce_gather_bf16(_dptr(slots), n_src, slot_rows, rows, cols, ld, arr,
                                         len(dst_ptrs), dst_row0, dst_ld, _stream(stream)),
           "b200_reduce_gather_bf16")


def reduce_residual_adaln_gather(slots, n_src: int, slot_rows: int, rows: int, cols: int,
                                 ld: int, x, gate, scale, dst_ptrs, dst_row0: int, dst_ld: int,
                                 rows_per_mod: int = None, mod_stride: int = 0,
                                 eps: float = 1e-6, stream=None):
    """b200_reduce_residual_adaln_gather: sum the first `rows` rows of n_src bf16 slots,
    x[:rows] += tanh(gate) * sum (f32 x, this owner's rows of the residual stream), then
    bf16(LN(x) * (1 + scale)) broadcast to dst_ptrs at row dst_row0.  gate / scale: f32
    [n_mod, cols] rows mod_stride apart (one row for every token when rows_per_mod is
    None)."""
    arr = _ptr_array(dst_ptrs)
    if rows_per_mod is None:
        rows_per_mod = 1 << 62
    _check(lib().b200_reduce_residual_adaln_gather(
        _dptr(slots), n_src, slot_rows, rows, cols, ld, _dptr(x), x.stride(0), _dptr(gate),
        _dptr(scale), rows_per_mod, mod_stride, float(eps), arr, len(dst_ptrs), dst_row0,
        dst_ld, _stream(stream)), "b200_reduce_residual_adaln_gather")


KQUANT_TYPES = {"q4_k": 0, "q6_k": 1}
KQUANT_GEMV_MAX_ROWS = 2


def kquant_gemv(x, blocks, qtype: str, n: int, out=None, stream=None):
    """b200_kquant_gemv: x f32 [m, k] (m <= 2) times the k-quant weight [n, k] (GGUF
    super-blocks, uint8 [n, k / 256 * block bytes]) transposed -> f32 [m, n]."""
    import torch
    m, k = x.shape
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    _check(lib().b200_kquant_gemv(_dptr(x), x.stride(0), _dptr(blocks), KQUANT_TYPES[qtype],
                                  _dptr(out), out.stride(0), m, n, k, _stream(stream)),
           "b200_kquant_gemv")
    return out


def reduce_nvls(mc_part: int, part_ld: int, mc_out: int, out_ld: int, row0: int, rows: int,
                cols: int, x=None, gate=None, scale=None, rows_per_mod: int = None,
                mod_stride: int = 0, eps: float = 1e-6, stream=None):
    """b200_reduce_nvls: rows [row0, row0 + rows) of every rank's partial summed by the
    NVSwitch (multicast addresses mc_part / mc_out, ints), optionally x += tanh(gate) * sum
    and LN(x) * (1 + scale) (x: this owner's f32 rows), written to every rank's output."""
    if rows_per_mod is None:
        rows_per_mod = 1 << 62
    _check(lib().b200_reduce_nvls(
        mc_part, part_ld, mc_out, out_ld, row0, rows, cols, _dptr(x),
        0 if x is None else x.stride(0), _dptr(gate), _dptr(scale), rows_per_mod, mod_stride,
        float(eps), _stream(stream)), "b200_reduce_nvls")


def qkv_norm_rope_gemm(x, w_qkv, batch: int, tokens: int, heads: int, norm_q_w, norm_k_w, pe,
                       eps: float = 1e-6, q_rot=None, k_rot=None, v=None, status=None,
                       stream=None):
    """x bf16 [B*T, C] @ w_qkv[3*H*128, C]^T with the Q/K RMSNorm + RoPE in the epilogue ->
    (q_rot, k_rot) head-major bf16 [B, H, T, 128] and v token-major bf16 [B, T, H, 128].
    pe f32 [T, 128] (shared) or [B, T, 128] (one table per batch row)."""
    import torch
    dev = x.device
    if q_rot is None:
        q_rot = torch.empty((batch, heads, tokens, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    if k_rot is None:
        k_rot = torch.empty((batch, heads, tokens, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    if v is None:
        v = torch.empty((batch, tokens, heads, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    pe_bs = pe.shape[-2] * pe.shape[-1] if pe.dim() == 3 else 0
    _check(lib().b200_qkv_norm_rope_gemm(_dptr(x), x.stride(0), _dptr(w_qkv), batch, tokens, heads,
                                         x.shape[1], _dptr(norm_q_w), _dptr(norm_k_w), float(eps),
                                         _dptr(pe), pe_bs, _dptr(q_rot), _dptr(k_rot), _dptr(v),
                                         _dptr(status), _stream(stream)), "b200_qkv_norm_rope_gemm")
    return q_rot, k_rot, v


# ----------------------------------------------------------------- head-sharding communicator
TP_ID_BYTES = 128  # B200_TP_ID_BYTES
DTYPE_BF16, DTYPE_F32, DTYPE_F16 = 0, 1, 2  # b200_dtype


def tp_unique_id() -> bytes:
    """A new group id (b200_tp_unique_id), made on one rank and handed to the others."""
    buf = (ctypes.c_uint8 * TP_ID_BYTES)()
    _check(lib().b200_tp_unique_id(buf), "b200_tp_unique_id")
    return bytes(buf)


class TpComm:
    """The b200_tp.h communicator of a head-sharded group: the per-block sum of the
    `to_out` partials (b200_tp_out_proj_allreduce) on the caller's stream, with every host
    wait bounded by ``timeout_ms``."""

    def __init__(self, uid: bytes, world: int, rank: int, timeout_ms: int = 60000):
        if len(uid) != TP_ID_BYTES:
            raise ValueError(f"group id must be {TP_ID_BYTES} bytes")
        h = ctypes.c_void_p()
        ub = (ctypes.c_uint8 * TP_ID_BYTES).from_buffer_copy(uid)
        _check(lib().b200_tp_init(ctypes.byref(h), ub, world, rank, timeout_ms), "b200_tp_init")
        self._h = h

    @classmethod
    def from_group(cls, group=None, timeout_ms: int = 60000):
        """Every rank of a torch.distributed group (any backend) calls this; rank 0's id
        reaches the others by broadcast."""
        import torch.distributed as dist
        obj = [tp_unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0,
                                   group=group)
        return cls(obj[0], dist.get_world_size(group), dist.get_rank(group), timeout_ms)

    @property
    def rank(self) -> int:
        return lib().b200_tp_rank(self._h)

    @property
    def size(self) -> int:
        return lib().b200_tp_size(self._h)

    def allreduce_(self, t, stream=None):
        """In-place sum over the group of a contiguous bf16 or f32 device tensor."""
        import torch
        if not t.is_contiguous():
            raise ValueError("partial must be contiguous")
        dt = {torch.bfloat16: DTYPE_BF16, torch.float32: DTYPE_F32}.get(t.dtype)
        if dt is None:
            raise ValueError("partial must be bf16 or f32")
        _check(lib().b200_tp_out_proj_allreduce(self._h, _dptr(t), t.numel(), dt, _stream(stream)),
               "b200_tp_out_proj_allreduce")
        return t

    def wait(self, stream=None):
        _check(lib().b200_tp_wait(self._h, _stream(stream)), "b200_tp_wait")

    def close(self):
        if self._h:
            h, self._h = self._h, None
            _check(lib().b200_tp_destroy(h), "b200_tp_destroy")
