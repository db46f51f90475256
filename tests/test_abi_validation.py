"""CPU: every entry point of `include/hb_b200.h` checks its arguments on the host and returns the documented
status before it touches the device, so these calls run without a GPU. Pointers are stand-in addresses
(16-byte aligned unless a case misaligns one on purpose); each case fails a check that comes before the
first CUDA call of its entry point, so no address is ever dereferenced. The reference raises `ValueError`
at trace time for unsupported shapes (`dense_attention.py:119-120`, `band_attention.py:138-140`); here the
C ABI returns HB_ERR_SHAPE and `_lib.call` turns it into `ValueError`."""
import ctypes

import pytest

from hummingbird_b200 import _lib

P = 0x7F0000001000      # stand-in device address, 16-byte aligned, never dereferenced
MIS = P + 4             # not 8- or 16-byte aligned
TILE = 128 * 64 * 2     # one prepared 128 x 64 bf16 tile


@pytest.fixture(scope="module")
def lib():
    from hummingbird_b200 import build
    build.build()
    return _lib.lib()


def _prep_bytes(batch, rows, heads):
    return batch * heads * 5 * -(-rows // 128) * TILE


def test_version_and_workspace_queries(lib):
    assert lib.hb_version() == 100
    n = ctypes.c_size_t(0)
    assert lib.hb_dense_workspace_bytes(1, 646, 8, ctypes.byref(n)) == _lib.HB_OK
    assert n.value == _prep_bytes(1, 646, 16)           # config 1: 6 row tiles x 16 heads x 5 sections
    assert lib.hb_dense_workspace_bytes(2, 2648, 8, ctypes.byref(n)) == _lib.HB_OK
    assert n.value == _prep_bytes(2, 2648, 16)
    assert lib.hb_band_workspace_bytes(1, 82688, 4, 128, 16, ctypes.byref(n)) == _lib.HB_OK
    assert n.value == 0                                 # window <= 128: the fused band kernel needs no workspace
    assert lib.hb_band_workspace_bytes(1, 82688, 4, 129, 16, ctypes.byref(n)) == _lib.HB_OK
    assert n.value == _prep_bytes(1, 82688, 8)
    assert lib.hb_dense_workspace_bytes(0, 646, 8, ctypes.byref(n)) == _lib.HB_ERR_SHAPE
    assert lib.hb_dense_workspace_bytes(1, 646, 8, None) == _lib.HB_ERR_NULL
    assert lib.hb_dense_noalloc_max_bytes(ctypes.byref(n)) == _lib.HB_OK
    assert n.value == 64 << 20


def _dense(**kw):
    """Arguments of a valid config-1 call (B=1, L=646, 16 heads, full-head RoPE), with overrides."""
    a = dict(qkv=P, qkv_rs=5120, q_w=P, k_w=P, cos=P, sin=P, table_stride=64, vmask=P, mask_bs=646, mask_rs=1,
             lam=None, out=P, out_rs=1024, batch=1, length=646, heads=16, head_dim=64, half=32, eps=1e-6,
             pair_begin=0, pair_count=8, ws=P, ws_bytes=_prep_bytes(1, 646, 16), stream=None)
    a.update(kw)
    return list(a.values())


@pytest.mark.parametrize("override,status", [
    (dict(head_dim=128), _lib.HB_ERR_SHAPE),             # the reference requires head_dim 64
    (dict(heads=15), _lib.HB_ERR_SHAPE),                 # heads come in (A, B) pairs
    (dict(half=12), _lib.HB_ERR_SHAPE),                  # rotary half must be 8, 16, 24 or 32
    (dict(pair_begin=6, pair_count=3), _lib.HB_ERR_SHAPE),  # pair range past the last pair
    (dict(qkv_rs=5112), _lib.HB_ERR_SHAPE),              # row shorter than the five sections
    (dict(out_rs=512), _lib.HB_ERR_SHAPE),               # output row shorter than the computed pairs
    (dict(qkv=MIS), _lib.HB_ERR_ALIGN),
    (dict(out_rs=1028), _lib.HB_ERR_ALIGN),              # row stride not a multiple of 16 bytes
    (dict(ws=MIS), _lib.HB_ERR_ALIGN),
    (dict(ws_bytes=_prep_bytes(1, 646, 16) - 1), _lib.HB_ERR_WORKSPACE),
    (dict(ws=None), _lib.HB_ERR_WORKSPACE),
    (dict(qkv=None), _lib.HB_ERR_NULL),
    (dict(vmask=None), _lib.HB_ERR_NULL),
])
def test_dense_rejects(lib, override, status):
    assert lib.hb_dense_diff_attn(*_dense(**override)) == status


def test_dense_noalloc_refuses_oversize_before_device_work(lib):
    # config 5's DiT call (L = 8,248, 8 pairs) needs 85 MB of prepared tiles: more than the 64 MiB scratch
    args = _dense(length=8248)[:-3] + [None]
    assert lib.hb_dense_diff_attn_noalloc(*args) == _lib.HB_ERR_WORKSPACE
    assert lib.hb_dense_diff_attn_noalloc(*(_dense(batch=0)[:-3] + [None])) == _lib.HB_ERR_SHAPE


def test_dense_noalloc_boundary_and_argument_checks_before_device_work(lib):
    """The size limit is exact (a problem one row tile past 64 MiB is refused), and a problem that fits still has
    its arguments checked on the host before the scratch is looked up on the device: a NULL or misaligned
    pointer returns its own status with no GPU present."""
    cap = 64 << 20
    # one head pair: 10 prepared tiles per 128-row tile; 410 row tiles = 4,100 tiles > 4,096, 409 fit
    over = _dense(length=410 * 128, heads=2, pair_count=1, qkv_rs=640, out_rs=128)[:-3] + [None]
    assert _prep_bytes(1, 410 * 128, 2) > cap
    assert lib.hb_dense_diff_attn_noalloc(*over) == _lib.HB_ERR_WORKSPACE
    fits = dict(length=409 * 128, heads=2, pair_count=1, qkv_rs=640, out_rs=128)
    assert _prep_bytes(1, 409 * 128, 2) <= cap
    assert lib.hb_dense_diff_attn_noalloc(*(_dense(qkv=None, **fits)[:-3] + [None])) == _lib.HB_ERR_NULL
    assert lib.hb_dense_diff_attn_noalloc(*(_dense(out=None, **fits)[:-3] + [None])) == _lib.HB_ERR_NULL
    assert lib.hb_dense_diff_attn_noalloc(*(_dense(qkv=MIS, **fits)[:-3] + [None])) == _lib.HB_ERR_ALIGN
    assert lib.hb_dense_diff_attn_noalloc(*(_dense(half=12, **fits)[:-3] + [None])) == _lib.HB_ERR_SHAPE


def _band(**kw):
    """Arguments of a valid config-2 call (L = 82,688, 8 heads, window 128, partial RoPE), with overrides."""
    a = dict(qkv=P, qkv_rs=2560, q_norm=P, k_norm=P, inv_freq=P, half=16, lam=None, out=P, out_rs=512, batch=1,
             rows=82688, q_begin=0, q_count=82688, pos0=0, heads=8, head_dim=64, window=128, pair_begin=0,
             pair_count=4, ws=None, ws_bytes=0, stages=_lib.HB_STAGE_ALL, stream=None)
    a.update(kw)
    return list(a.values())


@pytest.mark.parametrize("override,status", [
    (dict(stages=0), _lib.HB_ERR_SHAPE),
    (dict(stages=4), _lib.HB_ERR_SHAPE),
    (dict(head_dim=32), _lib.HB_ERR_SHAPE),
    (dict(window=-1), _lib.HB_ERR_SHAPE),
    (dict(q_begin=1), _lib.HB_ERR_SHAPE),                # query range past the held rows
    (dict(pos0=(1 << 24) - 82687), _lib.HB_ERR_SHAPE),   # RoPE positions beyond 2^24
    (dict(half=40), _lib.HB_ERR_SHAPE),
    (dict(qkv=MIS), _lib.HB_ERR_ALIGN),
    (dict(out_rs=516), _lib.HB_ERR_ALIGN),
    (dict(window=129), _lib.HB_ERR_WORKSPACE),           # wide windows take the two-stage path and a workspace
    (dict(inv_freq=None), _lib.HB_ERR_NULL),
    (dict(out=None), _lib.HB_ERR_NULL),
])
def test_band_rejects(lib, override, status):
    assert lib.hb_band_diff_attn(*_band(**override)) == status


def test_band_prepare_stage_needs_no_output(lib):
    # the prepare stage alone writes only the workspace: a null output passes the checks, the missing
    # workspace of the wide-window path does not
    assert lib.hb_band_diff_attn(*_band(out=None, stages=_lib.HB_STAGE_PREPARE, window=200)) == \
        _lib.HB_ERR_WORKSPACE


def _proj(**kw):
    """Arguments of a valid config-2 front-end call (x (1, 82,688, 512), to_qkv (2560, 512), prepared), with
    overrides."""
    a = dict(x=P, ldx=512, pre=P, w=P, ldw=512, q_norm=P, k_norm=P, inv_freq=P, half=16, out=P, ldo=2560, batch=1,
             rows=82688, pos0=0, d_model=512, heads=8, head_dim=64, prepare=1, stream=None)
    a.update(kw)
    return list(a.values())


@pytest.mark.parametrize("override,status", [
    (dict(d_model=576, ldx=576, ldw=576), _lib.HB_ERR_SHAPE),   # x tile no longer fits in shared memory
    (dict(d_model=96, ldx=96, ldw=96), _lib.HB_ERR_SHAPE),      # not whole 64-column chunks
    (dict(heads=7), _lib.HB_ERR_SHAPE),
    (dict(head_dim=32), _lib.HB_ERR_SHAPE),
    (dict(half=12), _lib.HB_ERR_SHAPE),
    (dict(ldo=2552), _lib.HB_ERR_SHAPE),
    (dict(pos0=(1 << 24) - 82687), _lib.HB_ERR_SHAPE),
    (dict(x=MIS), _lib.HB_ERR_ALIGN),
    (dict(ldw=516), _lib.HB_ERR_ALIGN),
    (dict(x=None), _lib.HB_ERR_NULL),
    (dict(k_norm=None), _lib.HB_ERR_NULL),
])
def test_band_projection_rejects(lib, override, status):
    assert lib.hb_band_qkv_project(*_proj(**override)) == status


def test_band_projection_needs_no_norms_unprepared(lib):
    # prepare = 0 is the plain projection: the DyT / RoPE parameters may be absent. The null check of the norms
    # comes before the shape checks, so a call whose only other fault is a short output stride reports the shape
    # (with prepare = 1 the same call reports the missing norms)
    kw = dict(q_norm=None, k_norm=None, inv_freq=None, half=0, ldo=2552)
    assert lib.hb_band_qkv_project(*_proj(prepare=0, **kw)) == _lib.HB_ERR_SHAPE
    assert lib.hb_band_qkv_project(*_proj(prepare=1, **kw)) == _lib.HB_ERR_NULL


def _prepared(**kw):
    a = dict(qkv=P, qkv_rs=2560, lam=None, out=P, out_rs=512, batch=1, rows=82688, q_begin=0, q_count=82688,
             heads=8, head_dim=64, window=128, pair_begin=0, pair_count=4, stream=None)
    a.update(kw)
    return list(a.values())


@pytest.mark.parametrize("override,status", [
    (dict(window=129), _lib.HB_ERR_SHAPE),        # the prepared form exists for the fused kernel only
    (dict(q_count=82689), _lib.HB_ERR_SHAPE),
    (dict(pair_count=5), _lib.HB_ERR_SHAPE),
    (dict(qkv_rs=2550), _lib.HB_ERR_SHAPE),
    (dict(out=MIS), _lib.HB_ERR_ALIGN),
    (dict(qkv=None), _lib.HB_ERR_NULL),
])
def test_band_prepared_rejects(lib, override, status):
    assert lib.hb_band_diff_attn_prepared(*_prepared(**override)) == status


def _cross(**kw):
    """Arguments of a valid DiT cross-attention call (B=2, 2,648 queries, 128 context tokens, 16 heads)."""
    a = dict(q=P, q_rs=2048, kv=P, kv_rs=3072, q_w=P, k_w=None, lam=None, out=P, out_rs=1024, batch=2,
             q_len=2648, kv_len=128, heads=16, head_dim=64, eps=1e-6, stream=None)
    a.update(kw)
    return list(a.values())


@pytest.mark.parametrize("override,status", [
    (dict(kv_len=385), _lib.HB_ERR_SHAPE),               # at most three 128-key tiles resident
    (dict(kv_len=0), _lib.HB_ERR_SHAPE),
    (dict(heads=3, q_rs=384, kv_rs=576, out_rs=192, lam=P), _lib.HB_ERR_SHAPE),  # lambda per pair: even heads
    (dict(kv_rs=3064), _lib.HB_ERR_SHAPE),
    (dict(q_rs=2052), _lib.HB_ERR_ALIGN),
    (dict(kv=MIS), _lib.HB_ERR_ALIGN),
    (dict(out=None), _lib.HB_ERR_NULL),
    (dict(q_w=None), _lib.HB_ERR_NULL),
])
def test_cross_rejects(lib, override, status):
    assert lib.hb_cross_diff_attn(*_cross(**override)) == status


def _gemm(**kw):
    """Arguments of a valid config-3 GEMM1 (M = 2,584, K = 1,024, N = 4,096)."""
    a = dict(qx=P, ldqx=1024, sx=P, qw=P, ldqw=1024, sw=P, bias=None, out=P, ldo=4096, acc=None, ldacc=0,
             M=2584, N=4096, K=1024, stream=None)
    a.update(kw)
    return list(a.values())


@pytest.mark.parametrize("override,status", [
    (dict(N=4080), _lib.HB_ERR_SHAPE),                   # N a multiple of 32
    (dict(K=1016, ldqx=1016, ldqw=1016), _lib.HB_ERR_SHAPE),  # K a multiple of 16
    (dict(M=0), _lib.HB_ERR_SHAPE),
    (dict(ldo=4000), _lib.HB_ERR_SHAPE),
    (dict(acc=P, ldacc=4095), _lib.HB_ERR_SHAPE),
    (dict(ldqx=1032), _lib.HB_ERR_ALIGN),                # int8 rows start on 16-byte boundaries
    (dict(qw=P + 8), _lib.HB_ERR_ALIGN),
    (dict(acc=P + 8, ldacc=4096), _lib.HB_ERR_ALIGN),
    (dict(sw=None), _lib.HB_ERR_NULL),
])
def test_w8a8_gemm_rejects(lib, override, status):
    assert lib.hb_w8a8_gemm(*_gemm(**override)) == status


def test_w8a8_gemm_glu_rejects(lib):
    # qx, ldqx, sx, qw, ldqw, sw, bias, z, ldz, M, F, K, stream: the GLU width F comes in 128-column blocks
    ok = dict(qx=P, ldqx=1024, sx=P, qw=P, ldqw=1024, sw=P, bias=None, z=P, ldz=4096, M=5296, F=4096, K=1024, s=None)

    def call(**kw):
        a = dict(ok)
        a.update(kw)
        return lib.hb_w8a8_gemm_glu(*a.values())
    assert call(F=4032, ldz=4032) == _lib.HB_ERR_SHAPE
    assert call(ldz=4000) == _lib.HB_ERR_SHAPE
    assert call(K=1000, ldqx=1008, ldqw=1008) == _lib.HB_ERR_SHAPE
    assert call(qw=P + 8) == _lib.HB_ERR_ALIGN
    assert call(z=None) == _lib.HB_ERR_NULL


def test_quantiser_rejects(lib):
    assert lib.hb_quant_rows_int8(P, 1024, 2584, 12, P, 1024, P, None) == _lib.HB_ERR_SHAPE
    assert lib.hb_quant_rows_int8(P, 1024, 2584, 1024, P + 4, 1024, P, None) == _lib.HB_ERR_ALIGN
    assert lib.hb_quant_rows_int8(P, 1024, 2584, 1024, P, 1024, None, None) == _lib.HB_ERR_NULL


def test_glue_entry_points_reject(lib):
    # residual + RMSNorm: h, ldh, y, ldy, gate, scale, shift, ldc, local, local_row0, weight, x, ldx, rows,
    # rows_per_batch, d, eps, stream
    def res(**kw):
        a = dict(h=P, ldh=1024, y=P, ldy=1024, gate=P, scale=None, shift=None, ldc=6144, local=None, row0=0,
                 weight=P, x=P, ldx=1024, rows=5296, rpb=2648, d=1024, eps=1e-6, stream=None)
        a.update(kw)
        return lib.hb_dit_residual_norm(*a.values())
    assert res(d=1000, ldh=1000, ldy=1000, ldx=1000) == _lib.HB_ERR_SHAPE   # d a multiple of 256
    assert res(d=2304, ldh=2304, ldy=2304, ldx=2304, ldc=2304) == _lib.HB_ERR_SHAPE  # d at most 2,048
    assert res(y=None) == _lib.HB_ERR_SHAPE              # a gate scales y: no gate without y
    assert res(scale=P) == _lib.HB_ERR_NULL              # adaLN scale without shift
    assert res(weight=None) == _lib.HB_ERR_NULL          # a normed output needs the norm weight
    assert res(local=MIS) == _lib.HB_ERR_ALIGN
    # the int8 form: h, ldh, y, ldy, gate, scale, shift, ldc, local, row0, weight, q, ldq, qscale, rows, rpb, d, eps
    def res_q(**kw):
        a = dict(h=P, ldh=1024, y=P, ldy=1024, gate=P, scale=None, shift=None, ldc=6144, local=None, row0=0,
                 weight=P, q=P, ldq=1024, qs=P, rows=5296, rpb=2648, d=1024, eps=1e-6, stream=None)
        a.update(kw)
        return lib.hb_dit_residual_norm_int8(*a.values())
    assert res_q(qs=None) == _lib.HB_ERR_NULL             # int8 rows need their scales
    assert res_q(q=None) == _lib.HB_ERR_NULL
    assert res_q(weight=None) == _lib.HB_ERR_NULL
    assert res_q(q=P + 4) == _lib.HB_ERR_ALIGN
    assert res_q(ldq=1000) == _lib.HB_ERR_SHAPE
    # GLU: glu, ldg, rows, F, z, ldz, q, ldq, scale, stream
    assert lib.hb_glu_rows(P, 8192, 5296, 4096, P, 4096, P, 4096, P, None) == _lib.HB_ERR_NULL   # z or q, not both
    assert lib.hb_glu_rows(P, 8192, 5296, 4096, None, 0, P, 4096, None, None) == _lib.HB_ERR_NULL  # q needs scales
    assert lib.hb_glu_rows(P, 8190, 5296, 4096, P, 4096, None, 0, None, None) == _lib.HB_ERR_SHAPE
    assert lib.hb_glu_rows(P, 1 << 20, 8, 1 << 19, P, 1 << 19, None, 0, None, None) == _lib.HB_ERR_SHAPE
    assert lib.hb_glu_rows(MIS, 8192, 5296, 4096, P, 4096, None, 0, None, None) == _lib.HB_ERR_ALIGN
    # per-head RMSNorm: x, ldx, rows, heads, weight, eps, out, ldo, stream
    assert lib.hb_head_rms_norm(P, 1000, 5296, 16, P, 1e-6, P, 1024, None) == _lib.HB_ERR_SHAPE
    assert lib.hb_head_rms_norm(P, 1024, 5296, 16, MIS, 1e-6, P, 1024, None) == _lib.HB_ERR_ALIGN
    assert lib.hb_head_rms_norm(P, 1024, 5296, 16, None, 1e-6, P, 1024, None) == _lib.HB_ERR_NULL


def test_python_call_maps_status_to_exceptions(lib):
    with pytest.raises(ValueError):                      # HB_ERR_SHAPE, as the reference's trace-time check
        _lib.call("hb_cross_diff_attn", *_cross(kv_len=385))
    with pytest.raises(_lib.HbError) as e:
        _lib.call("hb_cross_diff_attn", *_cross(kv=MIS))
    assert e.value.code == _lib.HB_ERR_ALIGN and "misaligned" in str(e.value)
    with pytest.raises(_lib.HbError) as e:
        _lib.call("hb_dense_diff_attn", *_dense(ws=None))
    assert e.value.code == _lib.HB_ERR_WORKSPACE
