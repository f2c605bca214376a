"""Torch-tensor front of the C ABI: output/workspace allocation, pointer and stream passing.

PyTorch is used only as the owner of device memory and of the current CUDA stream; every
computation below runs in libcfk_b200.so.  Tensors must live on a CUDA device: there is no CPU path.
"""
import ctypes

import torch

from colabfold_kernels import _lib

_TAGS = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float8_e4m3fn: _lib.E4M3}


def tag(dtype):
  try:
    return _TAGS[dtype]
  except KeyError:
    raise TypeError(f"unsupported dtype {dtype}") from None


def _ptr(t):
  if t is None:
    return None
  if not t.is_cuda:
    raise ValueError("colabfold_kernels (B200) takes CUDA tensors only: there is no CPU fallback")
  return ctypes.c_void_p(t.data_ptr())


def _stream():
  return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _c(t):
  return None if t is None else t.contiguous()


def device_status(reset=True):
  """The per-device word kernels set when a bounded wait ran out (0 = clean)."""
  return _lib.load().cfk_last_device_status(int(reset))


# ------------------------------------------------------------------------------------------ LayerNorm
def layer_norm(x, scale, offset, eps=1e-5):
  x = _c(x)
  c = x.shape[-1]
  y = torch.empty_like(x)
  m = x.numel() // c
  with torch.cuda.device(x.device):
    _lib.call("cfk_layer_norm", _ptr(x), _ptr(_c(scale.float())), _ptr(_c(offset.float())), _ptr(y), m, c,
              tag(x.dtype), float(eps), _stream())
  return y


def layer_norm_bwd(x, scale, dy, eps=1e-5):
  x, dy = _c(x), _c(dy.to(x.dtype))
  c = x.shape[-1]
  m = x.numel() // c
  dx = torch.empty_like(x)
  dscale = torch.empty(c, dtype=torch.float32, device=x.device)
  doffset = torch.empty(c, dtype=torch.float32, device=x.device)
  with torch.cuda.device(x.device):
    nbytes = _lib.load().cfk_layer_norm_bwd_workspace_bytes(m, c)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _lib.call("cfk_layer_norm_bwd", _ptr(x), _ptr(_c(scale.float())), _ptr(dy), _ptr(dx), _ptr(dscale), _ptr(doffset),
              m, c, tag(x.dtype), float(eps), _ptr(ws), nbytes, _stream())
  return dx, dscale, doffset


# ------------------------------------------------------------------------------------------ attention
def attention_fwd(q, k, v, bias, kmask, scale, seq_major=False, want_lse=False):
  """q/k/v [n,h,s,d] (or [n,s,h,d]); bias [h,sq,sk] or None; kmask [n,sk] bool/uint8 -> out (, lse [n,h,sq])."""
  q, k, v = _c(q), _c(k), _c(v)
  if seq_major:
    n, sq, h, d = q.shape
    sk = k.shape[1]
  else:
    n, h, sq, d = q.shape
    sk = k.shape[2]
  bias = None if bias is None else _c(bias.to(q.dtype))
  km = _c(kmask.to(torch.uint8))
  out = torch.empty_like(q)
  lse = torch.empty((n, h, sq), dtype=torch.float32, device=q.device) if want_lse else None
  with torch.cuda.device(q.device):
    _lib.call("cfk_attention_fwd", _ptr(q), _ptr(k), _ptr(v), _ptr(bias), _ptr(km), _ptr(out), _ptr(lse), n, h, sq, sk,
              d, tag(q.dtype), int(seq_major), float(scale), _stream())
  return (out, lse) if want_lse else out


def attention_bwd(q, k, v, bias, kmask, out, dout, lse, scale, seq_major=False, want_dbias=True):
  """-> dq, dk, dv, dbias [h,sq,sk] fp32 (None when not wanted)."""
  q, k, v, out = _c(q), _c(k), _c(v), _c(out)
  dout = _c(dout.to(q.dtype))
  if seq_major:
    n, sq, h, d = q.shape
    sk = k.shape[1]
  else:
    n, h, sq, d = q.shape
    sk = k.shape[2]
  bias = None if bias is None else _c(bias.to(q.dtype))
  km = _c(kmask.to(torch.uint8))
  dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
  dbias = torch.empty((h, sq, sk), dtype=torch.float32, device=q.device) if want_dbias else None
  with torch.cuda.device(q.device):
    nbytes = _lib.load().cfk_attention_bwd_workspace_bytes(n, h, sq, sk, d, tag(q.dtype))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    _lib.call("cfk_attention_bwd", _ptr(q), _ptr(k), _ptr(v), _ptr(bias), _ptr(km), _ptr(out), _ptr(dout),
              _ptr(_c(lse)), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dbias), n, h, sq, sk, d, tag(q.dtype),
              int(seq_major), float(scale), _ptr(ws), nbytes, _stream())
  return dq, dk, dv, dbias


def trim_limits(kmask):
  km = _c(kmask.to(torch.uint8))
  lim = torch.empty(km.shape[0] + 1, dtype=torch.int32, device=km.device)
  with torch.cuda.device(km.device):
    _lib.call("cfk_trim_limits", _ptr(km), _ptr(lim), km.shape[0], km.shape[1], _stream())
  return lim


def packed_attention_fwd(p, bias, kmask, gate_bias, sm_scale, column=False, trim=False, want_lse=False, p8=None):
  """p [X,Y,G,H,D] -> out [X,Y,H,D] (, lse [batch,H,S]).
  p8 [X,Y,2,H,D] float8_e4m3fn: q (multiplied by sm_scale * log2(e) before rounding, the static scale
  fp8_attention_slots names) and k; p then holds the remaining slots v[, gate] and the scores run in e4m3."""
  p = _c(p)
  if p8 is not None:
    return _packed_attention_qk8(p, _c(p8), bias, kmask, gate_bias, column, trim, want_lse)
  x, y, g, h, d = p.shape
  nb, s = (y, x) if column else (x, y)
  bias = None if bias is None else _c(bias.to(p.dtype))
  gb = None if gate_bias is None else _c(gate_bias.to(p.dtype))
  km = _c(kmask.to(torch.uint8))
  out = torch.empty((x, y, h, d), dtype=p.dtype, device=p.device)
  lse = torch.empty((nb, h, s), dtype=torch.float32, device=p.device) if want_lse else None
  lim = trim_limits(km) if trim else None
  with torch.cuda.device(p.device):
    _lib.call("cfk_packed_attention_fwd", _ptr(p), _ptr(bias), _ptr(km), _ptr(gb), _ptr(out), _ptr(lse), _ptr(lim),
              x, y, g, h, d, tag(p.dtype), int(column), float(sm_scale), _stream())
  return (out, lse) if want_lse else out


def _packed_attention_qk8(p, p8, bias, kmask, gate_bias, column, trim, want_lse):
  x, y, g, h, d = p.shape
  if p8.dtype != torch.float8_e4m3fn or tuple(p8.shape) != (x, y, 2, h, d) or p.dtype != torch.bfloat16:
    raise ValueError("p8 must be float8_e4m3fn [X,Y,2,H,D] beside a bfloat16 p [X,Y,G,H,D]")
  nb, s = (y, x) if column else (x, y)
  bias = None if bias is None else _c(bias.to(p.dtype))
  gb = None if gate_bias is None else _c(gate_bias.to(p.dtype))
  km = _c(kmask.to(torch.uint8))
  out = torch.empty((x, y, h, d), dtype=p.dtype, device=p.device)
  lse = torch.empty((nb, h, s), dtype=torch.float32, device=p.device) if want_lse else None
  lim = trim_limits(km) if trim else None
  with torch.cuda.device(p.device):
    # q carries sm_scale * log2(e): the raw products are log2-domain logits, ln 2 brings them to the natural domain
    _lib.call("cfk_packed_attention_fwd_qk8", _ptr(p), _ptr(p8), _ptr(bias), _ptr(km), _ptr(gb), _ptr(out), _ptr(lse),
              _ptr(lim), x, y, g, h, d, int(column), float(0.6931471805599453), _stream())
  return (out, lse) if want_lse else out


# ------------------------------------------------------------------------------------------ peer all-to-all
def peer_alltoall(send, recv_ptrs, flag_ptrs, counter, rank, parts, rows=1, run_bytes=None, src_part=None, src_row=0,
                  dst_part=None, dst_row=0):
  """Part p of send into rank p's receive buffer (device pointers in recv_ptrs), then the flag barrier.  By default
  send is [parts, chunk]; with rows / run_bytes / strides (bytes) a part is `rows` strided runs on either side."""
  send = _c(send)
  chunk = send.numel() * send.element_size() // parts
  run_bytes = chunk if run_bytes is None else run_bytes
  src_part = chunk if src_part is None else src_part
  dst_part = chunk if dst_part is None else dst_part
  with torch.cuda.device(send.device):
    _lib.call("cfk_peer_alltoall", _ptr(send), _ptr(recv_ptrs), _ptr(flag_ptrs), _ptr(counter), int(rank), int(parts), int(rows),
              int(run_bytes), int(src_part), int(src_row), int(dst_part), int(dst_row), _stream())


# ------------------------------------------------------------------------------------------ contraction
def contract(a, b, alpha=1.0):
  """out[c,i,j] = alpha * sum_k a[c,i,k] b[c,j,k]; a, b bf16 or float8_e4m3fn -> bf16."""
  a, b = _c(a), _c(b)
  c, i, k = a.shape
  j = b.shape[1]
  out = torch.empty((c, i, j), dtype=torch.bfloat16, device=a.device)
  with torch.cuda.device(a.device):
    _lib.call("cfk_contract", _ptr(a), _ptr(b), _ptr(out), c, i, j, k, tag(a.dtype), float(alpha), _stream())
  return out


def contract_gathered(a, b_parts, alpha=1.0):
  """contract(a, b) with b given as [parts, c, j/parts, k], an all-gather's output, read in place -> [c, i, j] bf16."""
  a, b_parts = _c(a), _c(b_parts)
  c, i, k = a.shape
  parts, _, jp, _ = b_parts.shape
  out = torch.empty((c, i, parts * jp), dtype=torch.bfloat16, device=a.device)
  with torch.cuda.device(a.device):
    _lib.call("cfk_contract_gathered", _ptr(a), _ptr(b_parts), _ptr(out), c, i, parts * jp, k, tag(a.dtype), float(alpha), parts,
              _stream())
  return out


def contract_exchanged(a_parts, b_parts, split_k=False, alpha=1.0, out=None):
  """The contraction between two all-to-alls over the channel axis.  split_k False: a_parts [P, c, i/P, k],
  b_parts [P, c, j/P, k]; True: a_parts [P, c, i, k/P], b_parts [P, c, j, k/P] -> [P, c, i/P, j] bf16, the send buffer
  of the all-to-all back to row shards."""
  a_parts, b_parts = _c(a_parts), _c(b_parts)
  parts, c = a_parts.shape[0], a_parts.shape[1]
  if split_k:
    i, j, k = a_parts.shape[2], b_parts.shape[2], a_parts.shape[3] * parts
  else:
    i, j, k = a_parts.shape[2] * parts, b_parts.shape[2] * parts, a_parts.shape[3]
  if out is None:
    out = torch.empty((parts, c, i // parts, j), dtype=torch.bfloat16, device=a_parts.device)
  with torch.cuda.device(a_parts.device):
    _lib.call("cfk_contract_exchanged", _ptr(a_parts), _ptr(b_parts), _ptr(out), c, i, j, k, tag(a_parts.dtype), float(alpha),
              parts, int(split_k), _stream())
  return out


def contract_exchanged_peer(a_parts, b_parts, out_ptrs, rank, split_k=False, alpha=1.0):
  """contract_exchanged whose stores are the all-to-all back to row shards: out_ptrs is a list of P device addresses
  (ints), entry q = rank q's receive buffer [P, c, i/P, j] bf16; rows of part q land at index `rank` of buffer q.  The
  caller runs a barrier across the ranks before reading its own buffer."""
  import ctypes
  a_parts, b_parts = _c(a_parts), _c(b_parts)
  parts, c = a_parts.shape[0], a_parts.shape[1]
  if split_k:
    i, j, k = a_parts.shape[2], b_parts.shape[2], a_parts.shape[3] * parts
  else:
    i, j, k = a_parts.shape[2] * parts, b_parts.shape[2] * parts, a_parts.shape[3]
  op = (ctypes.c_void_p * parts)(*[int(v) for v in out_ptrs])
  with torch.cuda.device(a_parts.device):
    _lib.call("cfk_contract_exchanged_peer", _ptr(a_parts), _ptr(b_parts), op, int(rank), c, i, j, k, tag(a_parts.dtype),
              float(alpha), parts, int(split_k), _stream())


# ------------------------------------------------------------------------------------------ projection family
def _f32(t):
  return _c(t.float())


def gated_dual_proj(x, wp, bp, wg, bg, mask, split=False, channel_major=False, activation=0):
  """mask * (x wp + bp) * act(x wg + bg); bf16.  -> [m,p], or (left, right) each [m,p/2] / [p/2,m]."""
  x = _c(x)
  m, k = x.shape
  p = wp.shape[1]
  dt = x.dtype
  if split:
    shape = (p // 2, m) if channel_major else (m, p // 2)
    out0, out1 = torch.empty(shape, dtype=dt, device=x.device), torch.empty(shape, dtype=dt, device=x.device)
  else:
    out0, out1 = torch.empty((m, p), dtype=dt, device=x.device), None
  with torch.cuda.device(x.device):
    _lib.call("cfk_gated_dual_proj", _ptr(x), _ptr(_c(wp.to(dt))), _ptr(_c(bp.to(dt))), _ptr(_c(wg.to(dt))),
              _ptr(_c(bg.to(dt))), _ptr(_c(mask.to(dt))), _ptr(out0), _ptr(out1), m, k, p, int(split),
              int(channel_major), int(activation), _stream())
  return (out0, out1) if split else out0


def ln_gated_dual_proj(x, ln_scale, ln_offset, wp, bp, wg, bg, mask, eps=1e-5, transpose=False, pad=1, fp8=False,
                       fp8_scale=1.0):
  """-> left, right channel-major: [p/2, m'] for x [m,k], [p/2, a, b'] / [p/2, b, a'] for the pair x [a,b,k].
  fp8 stores e4m3 of value * fp8_scale (per-tensor scale; contract(..., alpha=1 / scale**2) undoes it)."""
  if not fp8_scale > 0:
    raise ValueError("ln_gated_dual_proj: fp8_scale must be positive")
  x = _c(x)
  dt = x.dtype
  k, p = x.shape[-1], wp.shape[1]
  ci = p // 2
  if x.ndim == 3:
    a, b = x.shape[0], x.shape[1]
    outer, inner = (b, a) if transpose else (a, b)
    shape = (ci, outer, -(-inner // pad) * pad)
  else:
    a, b = x.shape[0], 0
    shape = (ci, -(-a // pad) * pad)
  odt = torch.float8_e4m3fn if fp8 else dt
  left, right = torch.empty(shape, dtype=odt, device=x.device), torch.empty(shape, dtype=odt, device=x.device)
  with torch.cuda.device(x.device):
    _lib.call("cfk_ln_gated_dual_proj", _ptr(x), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(wp.to(dt))),
              _ptr(_c(bp.to(dt))), _ptr(_c(wg.to(dt))), _ptr(_c(bg.to(dt))), _ptr(_c(mask.to(dt))), _ptr(left),
              _ptr(right), a, b, k, p, int(transpose), int(pad), int(fp8), float(fp8_scale), float(eps), _stream())
  return left, right


def ln_gated_dual_proj_peer(x, ln_scale, ln_offset, wp, bp, wg, bg, mask, left_ptrs, right_ptrs, rank, eps=1e-5,
                            transpose=False, pad=1):
  """ln_gated_dual_proj of the pair x [a,b,128] (bf16, 128 + 128 channels out) whose stores are the all-to-all over
  channels: left_ptrs / right_ptrs are lists of P device addresses (ints), entry q = rank q's receive buffer
  [P, 128 / P, outer, inner']; this rank's channel part q lands at index `rank` of buffer q.  Nothing is returned: the
  caller runs a barrier across the ranks (peer_alltoall with rows=0) before reading its own buffer."""
  import ctypes
  x = _c(x)
  dt = x.dtype
  parts = len(left_ptrs)
  lp = (ctypes.c_void_p * parts)(*[int(v) for v in left_ptrs])
  rp = (ctypes.c_void_p * parts)(*[int(v) for v in right_ptrs])
  with torch.cuda.device(x.device):
    _lib.call("cfk_ln_gated_dual_proj_peer", _ptr(x), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(wp.to(dt))),
              _ptr(_c(bp.to(dt))), _ptr(_c(wg.to(dt))), _ptr(_c(bg.to(dt))), _ptr(_c(mask.to(dt))), lp, rp, int(rank), parts,
              x.shape[0], x.shape[1], x.shape[2], wp.shape[1], int(transpose), int(pad), float(eps), _stream())


ln_gated_dual_proj_peer.dtypes = (torch.bfloat16,)


def _keep(keep):
  """keep [M] (the rows that matter, transition.py:29-38) -> (contiguous tensor or None, dtype tag)."""
  if keep is None:
    return None, 0
  keep = _c(keep.reshape(-1) if keep.dtype in (torch.float32, torch.bfloat16) else keep.reshape(-1).to(torch.float32))
  return keep, tag(keep.dtype)


def trimul_epilogue(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, residual=None, in_scale=None, in_offset=None,
                    eps=1e-5, add_input=False, out=None, keep=None):
  """(LN(x_cm^T) wo + bo) * sigmoid(g wg + bg) (+ residual | + act); g = act, or LN(act) when in_scale is given."""
  act = _c(act)
  x_cm = _c(x_cm if x_cm.dtype in (torch.bfloat16, torch.float32) else x_cm.to(torch.bfloat16))
  dt = act.dtype
  c, m = x_cm.shape
  ca, o = act.shape[1], wo.shape[1]
  if out is None:
    out = torch.empty((m, o), dtype=dt, device=act.device)
  res = None if residual is None else _c(residual.to(dt))
  kp, kt = _keep(keep)
  with torch.cuda.device(act.device):
    _lib.call("cfk_trimul_epilogue", _ptr(x_cm), tag(x_cm.dtype), _ptr(act),
              _ptr(None if in_scale is None else _f32(in_scale)), _ptr(None if in_offset is None else _f32(in_offset)),
              _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(wo.to(dt))), _ptr(_c(bo.to(dt))), _ptr(_c(wg.to(dt))),
              _ptr(_c(bg.to(dt))), _ptr(res), _ptr(kp), kt, _ptr(out), m, c, ca, o, float(eps), int(add_input), _stream())
  return out


def ln_projection(x, ln_scale, ln_offset, w=None, wb=None, eps=1e-5, f8=False, f8_scale=1.0, keep=None, f8_slots=(),
                  f8_scales=None):
  """-> (p [m, g*n] or None, bias [h, m] or None).
  f8_slots: those slots of w go, each times its static f8_scales entry, to a third output [m, len(f8_slots)*n] in
  e4m3 (saturating) and p keeps the others: -> (p, bias, p8), as packed_attn.py:234-305 returns them."""
  x = _c(x)
  dt = x.dtype
  m, a = x.shape
  p_out = b_out = None
  kp, kt = _keep(keep)
  if f8_slots:
    f8_slots = tuple(f8_slots)
    scales = tuple(f8_scales) if f8_scales else (1.0,) * len(f8_slots)
    rest = [g for g in range(w.shape[0]) if g not in f8_slots]
    # the static scale of a slot is folded into its weights (constants of the model), the kernel rounds with scale 1
    w8 = torch.stack([w[g].float() * sc for g, sc in zip(f8_slots, scales)]).to(dt)
    p8, _ = ln_projection(x, ln_scale, ln_offset, w8, None, eps=eps, f8=True, keep=keep)
    w_rest = torch.stack([w[g] for g in rest]) if rest else None  # views and a device copy: no host index tensor
    p_rest, b_out = ln_projection(x, ln_scale, ln_offset, w_rest, wb, eps=eps, keep=keep)
    return p_rest, b_out, p8
  with torch.cuda.device(x.device):
    if w is not None:
      g, _, n = w.shape
      p_out = torch.empty((m, g * n), dtype=torch.float8_e4m3fn if f8 else dt, device=x.device)
      _lib.call("cfk_ln_projection", _ptr(x), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(w.to(dt))),
                _ptr(kp), kt, _ptr(p_out), m, a, g, n, int(f8), float(f8_scale), float(eps), _stream())
    if wb is not None:
      h = wb.shape[1]
      hp = -(-h // 8) * 8
      wbp = torch.nn.functional.pad(wb.to(dt), (0, hp - h)).contiguous()
      b_out = torch.empty((h, m), dtype=dt, device=x.device)
      _lib.call("cfk_ln_head_bias", _ptr(x), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(wbp), _ptr(kp), kt,
                _ptr(b_out), m, a, h, hp, float(eps), _stream())
  return p_out, b_out


def output_projection(o, w, b, residual=None, out=None, keep=None):
  o = _c(o)
  dt = o.dtype
  m, k = o.shape
  c = w.shape[1]
  res = None if residual is None else _c(residual.to(dt))
  if out is None:
    out = torch.empty((m, c), dtype=dt, device=o.device)
  kp, kt = _keep(keep)
  with torch.cuda.device(o.device):
    _lib.call("cfk_output_projection", _ptr(o), _ptr(_c(w.to(dt))), _ptr(_c(b.to(dt))), _ptr(res), _ptr(kp), kt, _ptr(out),
              m, k, c, _stream())
  return out


def transition(x, ln_scale, ln_offset, w1, b1, w2, b2, keep=None, eps=1e-5, add_input=False):
  """relu(LN(x) w1 + b1) w2 + b2 (+ x) for x [..., c] (transition.py:100-146).  c = 128 or 256: one kernel of the
  library, both GEMMs on the tensor cores and the hidden activation on chip (cfk_transition).  c = 64: LayerNorm, the
  first GEMM, its bias and the relu are one kernel writing the hidden activation in bf16 and the second GEMM is the
  library GEMM.  keep: 128-row blocks it marks nowhere come out as zeros (x with add_input), as the reference leaves
  them; at c = 128 / 256 the kernel itself skips them."""
  shape = x.shape
  c, hdim = shape[-1], w1.shape[1]
  x2 = _c(x.reshape(-1, c))
  dt = x2.dtype
  m = x2.shape[0]
  kp, kt = _keep(None if keep is None else keep.reshape(-1))
  if c in (128, 256) and dt == torch.bfloat16 and hdim % (128 if c == 128 else 64) == 0:
    out = torch.empty_like(x2)  # blocks whose keep is negative throughout stay unwritten, as in the reference
    with torch.cuda.device(x2.device):
      _lib.call("cfk_transition", _ptr(x2), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(w1.to(dt))),
                _ptr(_c(b1.to(dt))), _ptr(_c(w2.to(dt))), _ptr(_c(b2.to(dt))), _ptr(kp), kt, _ptr(out), m, c, hdim,
                float(eps), int(add_input), _stream())
    return out.reshape(shape)
  h = torch.empty((m, hdim), dtype=dt, device=x2.device)
  with torch.cuda.device(x2.device):
    _lib.call("cfk_transition_hidden", _ptr(x2), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(w1.to(dt))),
              _ptr(_c(b1.to(dt))), _ptr(kp), kt, _ptr(h), m, c, hdim, float(eps), _stream())
  out = torch.addmm(b2.to(dt), h, w2.to(dt))
  if add_input:
    out.add_(x2)
  if keep is not None:
    pad = (-m) % 128
    rows = torch.nn.functional.pad(keep.reshape(-1) > 0, (0, pad)).view(-1, 128).any(1).repeat_interleave(128)[:m]
    out = torch.where(rows[:, None], out, x2 if add_input else torch.zeros_like(out))
  return out.reshape(shape)


def opm_projection(x, ln_scale, ln_offset, lw, lb, rw, rb, mask, eps=1e-5):
  x = _c(x)
  dt = x.dtype
  c, k = x.shape[-1], lw.shape[1]
  m = x.numel() // c
  left = torch.empty(x.shape[:-1] + (k,), dtype=dt, device=x.device)
  right = torch.empty_like(left)
  with torch.cuda.device(x.device):
    _lib.call("cfk_opm_projection", _ptr(x), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(lw.to(dt))),
              _ptr(_c(lb.to(dt))), _ptr(_c(rw.to(dt))), _ptr(_c(rb.to(dt))), _ptr(_c(mask.to(dt))), _ptr(left),
              _ptr(right), m, c, k, float(eps), _stream())
  return left, right


def opm_finish(x, bias, norm, residual=None, eps=1e-3, out=None):
  """(x + bias) / (eps + norm[..., None]) + residual; x [..., f] bf16, norm [...] fp32."""
  x = _c(x)
  f = x.shape[-1]
  m = x.numel() // f
  if out is None:
    out = torch.empty_like(x)
  res = None if residual is None else _c(residual.to(x.dtype))
  with torch.cuda.device(x.device):
    _lib.call("cfk_opm_finish", _ptr(x), _ptr(_c(bias.to(x.dtype))), _ptr(_f32(norm)), _ptr(res), _ptr(out), m, f,
              float(eps), _stream())
  return out


def _outer_product(left, right, fp8=False):
  """sum_s left[s,i,c] right[s,j,e] -> [i*j, c*e] bf16, rounded as the reference's opm_outer writes it (opm.py:124-134).
  fp8: the two projections are cast to e4m3 (saturating, unscaled) and the sum runs on the 8-bit tensor-core path."""
  s, ri, c = left.shape
  rj, e = right.shape[1], right.shape[2]
  a = left.permute(1, 2, 0).reshape(1, ri * c, s)       # [(i,c), s]
  b = right.permute(1, 2, 0).reshape(1, rj * e, s)      # [(j,e), s]
  if fp8:
    a, b = (t.clamp(-448.0, 448.0).to(torch.float8_e4m3fn) for t in (a, b))
  a, b = a.contiguous(), b.contiguous()
  if c == 32 and e == 32 and (s * a.element_size()) % 16 == 0:
    # the kernel stores the product as [i, j, c, e] itself: no transposed copy of the 2*ri*rj*c*e-byte intermediate
    outer = torch.empty((1, ri * rj, c * e), dtype=torch.bfloat16, device=left.device)
    with torch.cuda.device(left.device):
      _lib.call("cfk_opm_outer_product", _ptr(a), _ptr(b), _ptr(outer), ri, rj, s, tag(a.dtype), _stream())
    return outer
  return contract(a, b).view(ri, c, rj, e).permute(0, 2, 1, 3).reshape(1, ri * rj, c * e).contiguous()


def opm_outer(left, right, w):
  """The outer product mean in AF2's own order (opm.py:147-168): left [rows, B, C], right [rows, D, E], w [C*E, F] ->
  [B, D, F] in left's dtype; the rows' outer product rounded to left's dtype, then w over (c, e)."""
  rows, bdim, c = left.shape
  ddim, e = right.shape[1], right.shape[2]
  if e == c and opm_fused_supported(c, w.shape[1], left.dtype) and right.dtype == left.dtype:
    # one kernel, the product never written (as the reference's kernel): the operands channel-major with the rows
    # contiguous (a copy of rows * (B + D) * C values), a unit normaliser and no bias turn the deep form into this one
    pitch = -(-rows // 8) * 8
    lcm = torch.zeros((c, bdim, pitch), dtype=left.dtype, device=left.device)
    rcm = torch.zeros((e, ddim, pitch), dtype=left.dtype, device=left.device)
    lcm[:, :, :rows] = left.permute(2, 1, 0)
    rcm[:, :, :rows] = right.permute(2, 1, 0)
    f = w.shape[1]
    out = torch.empty((bdim, ddim, f), dtype=left.dtype, device=left.device)
    norm = torch.ones((bdim, ddim), dtype=torch.float32, device=left.device)
    zero = torch.zeros(f, dtype=left.dtype, device=left.device)
    with torch.cuda.device(left.device):
      _lib.call("cfk_opm_fused", _ptr(lcm), _ptr(rcm), _ptr(_c(w.to(left.dtype))), _ptr(zero), _ptr(norm), None, _ptr(out),
                bdim, ddim, rows, pitch, c, f, 0.0, _stream())
    return out
  outer = _outer_product(left, right)
  wt = w.to(left.dtype).t().contiguous().view(1, w.shape[1], c * e)
  return contract(outer, wt).view(bdim, ddim, w.shape[1])


def opm_update(lhs, t, bias, norm, residual=None, eps=1e-3):
  """The shallow outer product mean's pair update (opm.py:93-119): lhs [B, K], t [K, D, F], bias [F], norm [B, D],
  residual [B, D, F] -> (lhs . t + bias) / (eps + norm) (+ residual), [B, D, F]."""
  bdim, k = lhs.shape
  ddim, f = t.shape[1], t.shape[2]
  dt = lhs.dtype
  tt = t.to(dt).reshape(k, ddim * f).t().contiguous().view(1, ddim * f, k)
  x = contract(_c(lhs).view(1, bdim, k), tt).view(bdim, ddim, f)
  return opm_finish(x, bias, norm, None if residual is None else residual.to(dt), eps)


def opm_projection_cm(x, ln_scale, ln_offset, lw, lb, rw, rb, mask, eps=1e-5):
  """opm_projection for the fused outer product mean: x [s, r, c], mask [s, r] -> left, right [k, r, pitch], channel-major
  with the MSA depth contiguous (pitch = s rounded up to 8, the tail zeros)."""
  x = _c(x)
  dt = x.dtype
  s, r, c = x.shape
  k = lw.shape[1]
  pitch = -(-s // 8) * 8
  left = torch.empty((k, r, pitch), dtype=dt, device=x.device)
  right = torch.empty((k, r, pitch), dtype=dt, device=x.device)
  with torch.cuda.device(x.device):
    _lib.call("cfk_opm_projection_cm", _ptr(x), _ptr(_f32(ln_scale)), _ptr(_f32(ln_offset)), _ptr(_c(lw.to(dt))),
              _ptr(_c(lb.to(dt))), _ptr(_c(rw.to(dt))), _ptr(_c(rb.to(dt))), _ptr(_c(mask.to(dt))), _ptr(left), _ptr(right),
              s, r, c, k, pitch, float(eps), _stream())
  return left, right


def opm_fused_supported(c, f, dtype):
  """What cfk_opm_fused takes: 32-channel bf16 projections and 128 output channels."""
  return c == 32 and f == 128 and dtype == torch.bfloat16


def outer_product_mean_cm(left_cm, right_cm, mask_left, mask_right, w, bias, residual=None, eps=1e-3):
  """Deep-MSA outer product mean in one kernel from the channel-major projections of opm_projection_cm: left_cm
  [c, ri, pitch], right_cm [c, rj, pitch], masks [s, ri] / [s, rj], w [c*c, f] -> [ri, rj, f].  The outer product stays on
  chip (rounded to bf16 before the output weights, as the reference's opm_outer rounds it, opm.py:124-134); the mask
  overlap count comes from a kernel of the library (cfk_opm_norm)."""
  left_cm, right_cm = _c(left_cm), _c(right_cm)
  dt = left_cm.dtype
  c, ri, pitch = left_cm.shape
  rj, f = right_cm.shape[1], w.shape[1]
  depth = mask_left.shape[0]
  if right_cm.shape[0] != c or right_cm.shape[2] != pitch or w.shape[0] != c * c or mask_right.shape[0] != depth:
    raise ValueError("outer_product_mean_cm: operand shapes disagree")
  ml = _c(mask_left if mask_left.dtype in (torch.float32, torch.bfloat16) else mask_left.float())
  mr = _c(mask_right.to(ml.dtype))
  norm = torch.empty((ri, rj), dtype=torch.float32, device=left_cm.device)
  out = torch.empty((ri, rj, f), dtype=dt, device=left_cm.device)
  res = None if residual is None else _c(residual.to(dt))
  with torch.cuda.device(left_cm.device):
    _lib.call("cfk_opm_norm", _ptr(ml), _ptr(mr), tag(ml.dtype), _ptr(norm), depth, ri, rj, _stream())
    _lib.call("cfk_opm_fused", _ptr(left_cm), _ptr(right_cm), _ptr(_c(w.to(dt))), _ptr(_c(bias.to(dt))), _ptr(norm), _ptr(res),
              _ptr(out), ri, rj, depth, pitch, c, f, float(eps), _stream())
  return out


def outer_product_mean(left, right, mask_left, mask_right, w, bias, residual=None, eps=1e-3, fp8=False):
  """Deep-MSA outer product mean from the masked projections left [s, ri, c], right [s, rj, c]: two tensor-core GEMMs
  (the outer product over the MSA depth, rounded to bf16 as the reference's opm_outer does, opm.py:124-134; then the
  output weights w [c*c, f]) and the normalising tail -> [ri, rj, f].  ri < rj when the pair is row-sharded.
  fp8: the opt-in e4m3 outer product (projections cast to e4m3, fp32 accumulation)."""
  ri, c = left.shape[1], left.shape[2]
  rj, e = right.shape[1], right.shape[2]
  outer = _outer_product(left, right, fp8=fp8)
  wt = w.to(left.dtype).t().contiguous().view(1, w.shape[1], c * e)
  x = contract(outer, wt).view(ri, rj, w.shape[1])
  norm = mask_left.float().t() @ mask_right.float()
  return opm_finish(x, bias, norm, residual, eps)
