"""The C-ABI library: it loads, exports every function include/*.h declares, and validates its
arguments on the host before touching a device. CPU only (no compute calls)."""
from __future__ import annotations

import ctypes as C

import numpy as np

import large_model_b200 as q


def test_library_exports_every_declared_symbol():
    L = q.lib()
    names = q.declared_functions()
    assert len(names) >= 12
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_q8_block_layout_matches_reference():
    # QmsQ8 is 44 bytes: float d, float ds, int16 s16[2], int8 q[32] (src/kernels.h:7-12)
    assert q.Q8_DTYPE.itemsize == 44
    assert [q.Q8_DTYPE.fields[f][1] for f in ("d", "ds", "s16", "q")] == [0, 4, 8, 12]


def _desc(**kw):
    base = dict(n_embd=512, n_expert=32, n_used=4, n_ff=256, gate_type=q.T_Q4_0, up_type=q.T_Q4_0,
                down_type=q.T_Q4_0, router=1, gate=1, up=1, down=1, src_on_device=0)
    base.update(kw)
    return q.MoeDesc(**base)


def _create(d):
    h = C.c_void_p()
    rc = q.lib().qms_cuda_moe_create(C.byref(d), C.byref(h))
    return rc, q.lib().qms_cuda_last_error().decode()


def test_create_validates_shapes_before_any_device_call():
    rc, msg = _create(_desc(n_embd=288))                 # not the integer fast path
    assert rc == q.EUNSUPPORTED and "256" in msg
    rc, msg = _create(_desc(n_ff=100))
    assert rc == q.EUNSUPPORTED
    rc, msg = _create(_desc(down_type=q.T_Q6_K))
    assert rc == q.EUNSUPPORTED and "types" in msg
    rc, msg = _create(_desc(n_used=40, n_expert=32))     # k > n_expert
    assert rc == q.EINVAL
    rc, msg = _create(_desc(router=None))
    assert rc == q.EINVAL


def test_kernel_calls_validate_arguments():
    L = q.lib()
    assert L.qms_cuda_quantize_q8(None, 32, 1, None, None) == q.EINVAL
    assert L.qms_cuda_quantize_q8(C.c_void_p(16), 33, 1, C.c_void_p(16), None) == q.EINVAL
    assert L.qms_cuda_matvec_q8(q.T_Q8_0, C.c_void_p(16), 4, 32, C.c_void_p(16), 1, C.c_void_p(16), None) == q.EUNSUPPORTED
    assert L.qms_cuda_matvec_q8(q.T_Q6_K, C.c_void_p(16), 4, 32, C.c_void_p(16), 1, C.c_void_p(16), None) == q.EINVAL
    assert L.qms_cuda_moe_forward(None, None, 1, None, None, None, None, None, None) == q.EINVAL
    assert L.qms_cuda_moe_experts(None, None, None, 4, None, None) == q.EINVAL
    assert L.qms_cuda_moe_experts_q8(None, None, None, 4, None, None) == q.EINVAL
    p = C.c_void_p(16)
    assert L.qms_cuda_sample(None, 10, 1.0, 0.9, 0, p, p, None) == q.EINVAL          # no logits
    assert L.qms_cuda_sample(p, 10, 1.0, 0.9, 0, None, p, None) == q.EINVAL           # tempered draw without a state
    assert L.qms_cuda_sample(p, 5000, 1.0, 0.9, 2000, p, p, None) == q.EUNSUPPORTED   # more than 1024 candidates


def test_init_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        return
    rc = q.lib().qms_cuda_init(0)
    assert rc == q.ENODEV
    assert q.lib().qms_cuda_last_error()


def test_declared_functions_cite_reference():
    text = (q.HEADER).read_text()
    for cite in ("src/kernels.h:15", "src/kernels.h:19", "src/kernels.h:21", "src/model.c:1032"):
        assert cite in text


def _model_desc(**kw):
    base = dict(n_layer=2, n_embd=512, n_head=8, n_head_kv=2, head_dim=64, n_expert=32, n_used=4, n_ff=256,
                vocab=4096, eps=1e-6, rope_base=1e6, ctx=64, embd_type=q.T_Q4_0, embd=16, out_norm=16,
                output_type=q.T_Q6_K, output=16, src_on_device=0)
    base.update(kw)
    return q.ModelDesc(**base)


def _model_create(d):
    h = C.c_void_p()
    rc = q.lib().qms_cuda_model_create(C.byref(d), C.byref(h))
    return rc, q.lib().qms_cuda_last_error().decode()


def test_model_create_validates_config_before_any_device_call():
    rc, msg = _model_create(_model_desc(head_dim=96))
    assert rc == q.EUNSUPPORTED and "head_dim" in msg
    rc, msg = _model_create(_model_desc(n_head=6, n_head_kv=4))      # n_head % n_head_kv (read_cfg's check)
    assert rc == q.EINVAL and "inconsistent" in msg
    rc, msg = _model_create(_model_desc(n_embd=288))
    assert rc == q.EUNSUPPORTED and "256" in msg
    rc, msg = _model_create(_model_desc(output_type=q.T_Q8_0))
    assert rc == q.EUNSUPPORTED and "output type" in msg
    rc, msg = _model_create(_model_desc(embd_type=7))
    assert rc == q.EUNSUPPORTED and "token_embd" in msg
    rc, msg = _model_create(_model_desc(embd=None))
    assert rc == q.EINVAL
    rc, msg = _model_create(_model_desc(ctx=0))
    assert rc == q.EINVAL


def test_model_calls_validate_arguments():
    L = q.lib()
    p = C.c_void_p(16)
    assert L.qms_cuda_forward(None, p, 1, 0, p, 0, None) == q.EINVAL
    assert L.qms_cuda_forward_dev(None, p, 1, p, p, 0, None) == q.EINVAL
    assert L.qms_cuda_decode_step(None, p, p, None, None) == q.EINVAL
    assert L.qms_cuda_forward_seq(None, 0, p, 1, 0, p, 0, None) == q.EINVAL
    assert L.qms_cuda_forward_batch(None, 1, p, p, p) == q.EINVAL
    assert L.qms_cuda_decode_batch(None, 1, p, p, None, None) == q.EINVAL
    assert L.qms_cuda_model_set_sequences(None, 2) == q.EINVAL
    assert L.qms_cuda_model_copy_sequence(None, 0, 1, 4) == q.EINVAL
    assert L.qms_cuda_model_set_kv_type(None, q.T_F16) == q.EINVAL
    assert L.qms_cuda_model_set_layer(None, 0, None) == q.EINVAL
    assert L.qms_cuda_model_reserve(None, 4) == q.EINVAL
    assert L.qms_cuda_model_status(None) == q.EINVAL
    assert L.qms_cuda_model_profile(None, 1, None) == q.EINVAL
    assert L.qms_cuda_model_device_bytes(None) == 0
    L.qms_cuda_model_free(None)                                     # no-op


def test_noalloc_route_validates_before_any_device_call():
    """qms_cuda_moe_route_noalloc refuses sizes beyond its fixed scratch before any CUDA call."""
    L = q.lib()
    p = C.c_void_p(256)
    assert L.qms_cuda_moe_route_noalloc(p, 128, 4096, 8, p, 65, p, p, None, None) == q.EINVAL   # T > 64
    assert "64" in L.qms_cuda_last_error().decode()
    assert L.qms_cuda_moe_route_noalloc(p, 128, 8192, 8, p, 1, p, p, None, None) == q.EINVAL    # n_embd > 4096
    assert L.qms_cuda_moe_route_noalloc(p, 128, 4000, 8, p, 1, p, p, None, None) == q.EINVAL    # n_embd % 256
    assert L.qms_cuda_moe_route_noalloc(p, 300, 4096, 8, p, 1, p, p, None, None) == q.EINVAL    # n_expert > 256
    assert L.qms_cuda_moe_route_noalloc(p, 128, 128, 8, p, 1, p, p, None, None) == q.EINVAL     # 2 X > E
    assert L.qms_cuda_moe_route_noalloc(None, 128, 4096, 8, p, 1, p, p, None, None) == q.EINVAL
    assert L.qms_cuda_moe_route_noalloc(p, 128, 4096, 8, p, 1, None, p, None, None) == q.EINVAL
    assert L.qms_cuda_moe_route_noalloc(C.c_void_p(260), 128, 4096, 8, p, 1, p, p, None, None) == q.EINVAL  # router alignment


def test_ep_calls_validate_before_any_device_call():
    """qms_cuda_ep_pack / qms_cuda_ep_combine refuse bad shapes, splits and pointers on the host."""
    L = q.lib()
    p = C.c_void_p(256)
    #                      xn sel T  K  E    X    N   cap send_x send_e slot err stream
    assert L.qms_cuda_ep_pack(p, p, 4, 4, 500, 32, 2, 16, p, p, p, None, None) == q.EINVAL       # n_embd % 32
    assert L.qms_cuda_ep_pack(p, p, 4, 4, 512, 32, 3, 16, p, p, p, None, None) == q.EUNSUPPORTED  # 32 experts over 3
    assert L.qms_cuda_ep_pack(p, p, 4, 4, 512, 130, 65, 16, p, p, p, None, None) == q.EUNSUPPORTED  # > 64 ranks
    assert L.qms_cuda_ep_pack(p, p, 4, 4, 512, 32, 2, 0, p, p, p, None, None) == q.EINVAL        # cap 0
    assert L.qms_cuda_ep_pack(p, p, -1, 4, 512, 32, 2, 16, p, p, p, None, None) == q.EINVAL      # T < 0
    assert L.qms_cuda_ep_pack(p, p, 1 << 29, 8, 512, 32, 2, 16, p, p, p, None, None) == q.EINVAL  # slots overflow
    assert L.qms_cuda_ep_pack(p, None, 4, 4, 512, 32, 2, 16, p, p, p, None, None) == q.EINVAL    # no sel
    assert L.qms_cuda_ep_pack(None, None, 0, 4, 512, 32, 2, 16, None, p, None, None, None) == q.EINVAL  # no send_x
    assert L.qms_cuda_ep_pack(p, p, 4, 4, 512, 32, 2, 16, C.c_void_p(258), p, p, None, None) == q.EINVAL  # alignment
    assert "aligned" in L.qms_cuda_last_error().decode()
    assert L.qms_cuda_ep_combine(None, p, p, 4, 4, 512, None, p, None) == q.EINVAL
    assert L.qms_cuda_ep_combine(p, p, p, 70000, 4, 512, None, p, None) == q.EINVAL              # T > 65535
    assert L.qms_cuda_ep_combine(p, p, p, 0, 4, 512, None, p, None) == q.OK                      # nothing to do
