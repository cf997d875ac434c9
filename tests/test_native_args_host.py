"""Argument checking of the C ABI, on a machine without a GPU.

Every case here is rejected by the entry point's own checks, which run
before the entry point touches the device (no launch, no CUDA call), so the
fake addresses below are never dereferenced.  Also the pure size helpers of
the packed-weight entry points, against their layout arithmetic."""

import ctypes

import pytest

from forgeml_b200 import _native

EINVAL, EUNSUPPORTED = 1, 2
F32, F16, BF16 = _native.FML_F32, _native.FML_F16, _native.FML_BF16
FAKE = 1 << 20  # 1024-byte aligned, never dereferenced


def _rejects(name, code, match, *args):
    with pytest.raises(_native.NativeError, match=match) as e:
        _native.call(name, *args)
    assert e.value.code == code


@pytest.mark.parametrize("n,k", [(1, 1), (128, 64), (129, 64), (2048, 2048), (6144, 2048), (8192, 2048),
                                 (2048, 8192), (32000, 2048), (100, 70)])
def test_packed_weight_bytes_is_whole_16kb_tiles(n, k):
    lib = _native.load()
    # 128 weight rows x 128 bytes of K per tile, tiles padded on both axes
    want = -(-n // 128) * -(-(2 * k) // 128) * 16384
    assert lib.fml_packed_weight_bytes(n, k, BF16) == want
    assert lib.fml_packed_weight_bytes(n, k, F16) == want
    assert lib.fml_packed_weight_bytes(n, k, F32) == 0
    assert lib.fml_packed_weight_bytes(0, k, BF16) == 0
    assert lib.fml_packed_weight_bytes(n, -1, BF16) == 0


@pytest.mark.parametrize("n,k", [(1, 1), (64, 3), (512, 2048), (2048, 8191), (3, 5)])
def test_gemm_packed_b_bytes_is_the_3xtf32_image(n, k):
    lib = _native.load()
    kp = -(-k // 4) * 4  # K padded to 16 bytes of fp32
    want = -(-(n * 3 * kp * 4) // 256) * 256  # hi | lo | hi, 256-byte multiple
    assert lib.fml_gemm_packed_b_bytes(n, k, F32) == want
    assert lib.fml_gemm_packed_b_bytes(n, k, BF16) == 0
    assert lib.fml_gemm_packed_b_bytes(0, k, F32) == 0


def test_pack_weight_argument_checks():
    _rejects("fml_pack_weight", EUNSUPPORTED, "16-bit weights only", FAKE, 64, 128, 64, F32, FAKE, None)
    _rejects("fml_pack_weight", EINVAL, "null pointer", None, 64, 128, 64, BF16, FAKE, None)
    _rejects("fml_pack_weight", EINVAL, "bad shape", FAKE, 32, 128, 64, BF16, FAKE, None)  # ldw < k
    _rejects("fml_pack_weight", EINVAL, "1024-byte aligned", FAKE, 64, 128, 64, BF16, FAKE + 16, None)


def test_gemm_pack_b_argument_checks():
    need = _native.load().fml_gemm_packed_b_bytes(64, 32, F32)
    _rejects("fml_gemm_pack_b", EUNSUPPORTED, "fp32 only", FAKE, 64, 1, 32, 64, BF16, FAKE, need, None)
    _rejects("fml_gemm_pack_b", EINVAL, "null pointer", FAKE, 64, 1, 32, 64, F32, None, need, None)
    _rejects("fml_gemm_pack_b", EINVAL, "must be positive", FAKE, 64, 1, 0, 64, F32, FAKE, need, None)
    _rejects("fml_gemm_pack_b", EINVAL, "256-byte aligned", FAKE, 64, 1, 32, 64, F32, FAKE + 16, need, None)
    _rejects("fml_gemm_pack_b", EINVAL, "smaller than", FAKE, 64, 1, 32, 64, F32, FAKE, need - 256, None)


def test_gemm_packed_b_argument_checks():
    def call(dtype=F32, b_packed=FAKE):
        # a, lda_m, lda_k, b_packed, bias, bias_stride, residual, ldr, c, ldc, m, n, k, dtype, act, cfg,
        # workspace, workspace_bytes, stream
        _native.call("fml_gemm_packed_b", FAKE, 32, 1, b_packed, None, 0, None, 0, FAKE, 64, 16, 64, 32, dtype, 0,
                     None, None, 0, None)
    with pytest.raises(_native.NativeError, match="fp32 only") as e:
        call(dtype=BF16)
    assert e.value.code == EUNSUPPORTED
    with pytest.raises(_native.NativeError, match="256-byte aligned") as e:
        call(b_packed=FAKE + 16)
    assert e.value.code == EINVAL


def test_linear_packed_argument_checks():
    def call(dtype=BF16, act=0, ldo=256, packed=FAKE, m=8):
        _native.call("fml_linear_packed", FAKE, 128, packed, 256, 128, None, 0, None, 0, FAKE, ldo, m, dtype, act,
                     None, None)
    for kw, code, match in (({"dtype": F32}, EUNSUPPORTED, "16-bit only"), ({"act": 3}, EINVAL, "bad act"),
                            ({"ldo": 255}, EINVAL, "leading dimension"), ({"m": 0}, EINVAL, "must be positive"),
                            ({"packed": FAKE + 512}, EINVAL, "1024-byte aligned")):
        with pytest.raises(_native.NativeError, match=match) as e:
            call(**kw)
        assert e.value.code == code


def test_linear_fused_argument_checks():
    def call(fz, dtype=BF16, m=8, packed=FAKE, n=256):
        _native.call("neb_linear_fused", FAKE, 128, packed, n, 128, None, 0, FAKE, n, m, dtype, 0,
                     ctypes.byref(fz) if fz is not None else None, None)
    plain = _native.neb_fusion()
    for kw, code, match in (({"dtype": F32}, EUNSUPPORTED, "16-bit only"), ({"m": 33}, EUNSUPPORTED, "32 tokens"),
                            ({"packed": FAKE + 64}, EINVAL, "1024-byte aligned")):
        with pytest.raises(_native.NativeError, match=match) as e:
            call(plain, **kw)
        assert e.value.code == code
    with pytest.raises(_native.NativeError, match="null fusion descriptor"):
        call(None)
    both = _native.neb_fusion(ln_gamma=FAKE, ln_beta=FAKE, ln_wsum=FAKE)
    with pytest.raises(_native.NativeError, match="not both"):
        call(both)
    no_beta = _native.neb_fusion(ln_gamma=FAKE)
    with pytest.raises(_native.NativeError, match="gamma and beta"):
        call(no_beta)
    # KV epilogue: n must be q_cols + 2 * kv_heads * head_dim
    kv = _native.neb_fusion(k_pool=FAKE, v_pool=FAKE, slot_of=FAKE, start_pos=FAKE, q_cols=128, kv_heads=1,
                            head_dim=32, max_seq=64, tq=1)
    with pytest.raises(_native.NativeError, match="KV epilogue shape") as e:
        call(kv, n=256)
    assert e.value.code == EINVAL
    kv.v_pool = None
    with pytest.raises(_native.NativeError, match="KV epilogue pointers"):
        call(kv, n=192)
