"""Host logic of the selector surface, no GPU needed: the reference's selectors return a callable or None (the caller
then runs its own path) for the same reasons (fused_ops.py:43-64,221-323; asserted in tests/test_ln_fusions.py:77-125 of
the reference), and the library refuses to run without a CUDA device instead of falling back."""
import pytest
import torch

from colabfold_kernels import _lib, device, fused_ops

ON = {"use_pallas": True, "kernel_backend": "b200", "compute_capability": 100}
OFF = {"use_pallas": False}
bf = torch.bfloat16


def test_dispatch_has_the_reference_keys():
  cfg = device.dispatch()
  assert {"use_pallas", "kernel_backend"} <= set(cfg)
  assert device.is_rocm() is False


def test_everything_is_off_without_use_pallas():
  for sel, args in ((fused_ops.attention, (bf, 32, 32)), (fused_ops.layer_norm, (bf,)), (fused_ops.gated_dual_proj, (bf, 128)),
                    (fused_ops.ln_projection, (bf, 128)), (fused_ops.output_projection, (bf, 128, 128))):
    assert sel(OFF, *args) is None
  assert fused_ops.attention({"use_pallas": True, "kernel_backend": "cuda_legacy"}, bf, 32, 32) is None


@pytest.mark.skipif(not _lib.available(), reason="library not built")
def test_supported_and_declined_shapes():
  assert callable(fused_ops.attention(ON, bf, 32, 32, layout="seq"))
  assert callable(fused_ops.attention(ON, "bfloat16", 32, 32))           # dtype given by name, as JAX/numpy would
  assert callable(fused_ops.attention(ON, torch.float32, 32, 32))        # fp32 runs the fp32-math kernels
  assert fused_ops.attention(ON, torch.float16, 32, 32) is None
  assert fused_ops.attention(ON, bf, 32, 64) is None                     # key_dim != value_dim
  assert callable(fused_ops.layer_norm(ON, bf)) and fused_ops.layer_norm(ON, torch.float16) is None
  assert callable(fused_ops.ln_projection(ON, bf, 128)) and fused_ops.ln_projection(ON, bf, 96) is None
  assert fused_ops.ln_projection(ON, bf, 128, 100) is None               # packed width must be a multiple of 64
  assert callable(fused_ops.output_projection(ON, bf, 128, 128)) and fused_ops.output_projection(ON, bf, 128, 12) is None
  assert callable(fused_ops.opm_projection(ON, bf, 256, 32)) and fused_ops.opm_projection(ON, bf, 256, 200) is None
  # ops this build leaves to the caller
  assert callable(fused_ops.transition(ON, bf, 128, 512)) and fused_ops.transition(ON, bf, 96, 512) is None
  assert fused_ops.transition(ON, bf, 128, 100) is None and fused_ops.glu_transition(ON, bf, 128, 512) is None
  # the shallow outer-product forms take the reference's own shape rules (opm.py:88-90,142-144)
  assert callable(fused_ops.opm_update(ON, bf, 64, 128)) and fused_ops.opm_update(ON, bf, 40, 128) is None
  assert callable(fused_ops.opm_outer(ON, bf, 16, 32, 32, 128)) and fused_ops.opm_outer(ON, bf, 8, 32, 32, 128) is None


@pytest.mark.skipif(torch.cuda.is_available() or not _lib.available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
  """Without a CUDA device a call fails loudly: there is no CPU path behind the selectors."""
  k = fused_ops.layer_norm(ON, torch.float32)
  x = torch.randn(4, 128)
  with pytest.raises(Exception):
    k(x, torch.ones(128), torch.zeros(128))


def test_status_names_cover_the_header():
  assert _lib.STATUS_NAMES[0] == "CFK_OK" and _lib.STATUS_NAMES[-8] == "CFK_ERR_UNSUPPORTED"
  assert "cfk_opm_outer_product" in _lib.PROTOTYPES and "cfk_layer_norm_bwd_static" in _lib.PROTOTYPES


def test_fp8_attention_slots_follow_the_reference_rules():
  """fused_ops.py:75-97 and tests/test_ln_fusions.py:162-172 of the reference: e4m3 slots only when global_config.fp8
  asks, never below the 8-bit MMA's K of 32, q (with its static scale sm_scale * log2 e) and k where the q.k kernel
  runs, and the k/v form is then not offered."""
  on = {**ON, "fp8": True}
  slots, scales = fused_ops.fp8_attention_slots(on, bf, 32, 264)
  assert slots == (0, 1) and scales[1] == 1.0 and abs(scales[0] - 32 ** -0.5 * 1.4426950408889634) < 1e-12
  assert fused_ops.fp8_attention_slots(on, None, 32, 0) is not None  # dtype None: "would any dtype do" (fused_ops.py:80)
  for d in (8, 16, 48, 64):
    assert fused_ops.fp8_attention_slots(on, bf, d, 64) is None
  assert fused_ops.fp8_attention_slots(ON, bf, 32, 64) is None
  assert fused_ops.fp8_attention_slots(on, torch.float32, 32, 64) is None
  assert fused_ops.fp8_attention(on, 32) is False and fused_ops.fp8_attention(on, 16) is False


def test_reference_restatement_of_the_e4m3_projection_slots():
  """ref_ln_projection with f8_slots returns (other slots, bias, chosen slots times their scales), packed_attn.py:308-318."""
  from colabfold_kernels import reference
  g = torch.Generator().manual_seed(0)
  x, w, wb = torch.randn(9, 64, generator=g), torch.randn(4, 64, 16, generator=g), torch.randn(64, 2, generator=g)
  sc, of = torch.ones(64), torch.zeros(64)
  p, b = reference.ref_ln_projection(x, sc, of, w, wb)
  ph, b2, p8 = reference.ref_ln_projection(x, sc, of, w, wb, f8_slots=(0, 1), f8_scales=(0.25, 1.0))
  p = p.reshape(9, 4, 16)
  assert torch.equal(b, b2)
  assert torch.allclose(ph.reshape(9, 2, 16), p[:, 2:]) and torch.allclose(p8.reshape(9, 2, 16)[:, 0], 0.25 * p[:, 0])
  assert torch.allclose(p8.reshape(9, 2, 16)[:, 1], p[:, 1])
