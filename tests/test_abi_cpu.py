"""CPU checks of the C ABI: the library loads without a GPU, exports every symbol the
header declares, and rejects bad arguments on the host before any launch."""
import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "fnx_b200.h"


def header_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fnx_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import build as fnx_build   # qwen-ascend_b200/build.py
    fnx_build.build()
    from fnx import _lib
    return _lib.lib()


def test_header_symbols_exported(lib):
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), s
    from fnx import _lib
    assert set(syms) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_version(lib):
    assert b"sm_100a" in lib.fnx_b200_version()


def test_host_side_rejections(lib):
    # rejected before any CUDA call, so these are safe without a device
    assert lib.fnx_weighted_reduce(None, None, None, None, 0, 10, 2560, 2560, 1, 0, None) == -1
    assert lib.fnx_weighted_reduce(None, None, None, None, 1, 10, 2560, 2560, 1, 1, None) == -1   # order != 0
    assert lib.fnx_weighted_reduce(None, None, None, None, 1, 10, 2560, 2560, 2, 0, None) == -1   # mode 2 w/o inverse
    assert lib.fnx_weighted_reduce(None, None, None, None, 1, 65, 2560, 2560, 1, 0, None) == -1
    assert lib.fnx_gather_pair(None, None, None, None, None, 0, 1, 1280, None) == -1
    assert lib.fnx_gather_pair(None, None, None, None, None, 16, 1, 1281, None) == -1
    assert lib.fnx_router_topk(None, 512, None, None, None, None, 4, 512, 33, None) == -1
    assert lib.fnx_router_topk(None, 100, None, None, None, None, 4, 512, 10, None) == -1
    assert lib.fnx_moe_permute(None, None, None, None, None, 10, 5000, None, 0, None) == -1
    assert lib.fnx_moe_permute(None, None, None, None, None, 10, 8, None, 0, None) == -5
    # grouped GEMM shape rules: K % 64, Nw % 128, epilogue in 0..4, act rows >= M without an index
    g = lib.fnx_moe_grouped_w4
    assert g(None, 2048, 64, None, 1, None, None, None, 1024, 8, 64, 100, 1024, 0, None) == -1
    assert g(None, 2048, 64, None, 1, None, None, None, 1024, 8, 64, 2048, 1000, 0, None) == -2
    assert g(None, 2048, 64, None, 1, None, None, None, 1024, 8, 64, 2048, 1024, 5, None) == -1
    assert g(None, 2048, 10, None, 1, None, None, None, 1024, 8, 64, 2048, 1024, 0, None) == -1  # rows < M
    # the expert-id form: an id table and E_w >= 1 required, epilogues 0-2 only, then the same rules
    gs = lib.fnx_moe_grouped_w4_sel
    assert gs(None, 2048, 64, None, 1, None, 8, None, None, None, 1024, 8, 64, 2048, 1024, 0, None) == -1
    assert gs(None, 2048, 64, None, 1, None, 0, 8, None, None, 1024, 8, 64, 2048, 1024, 0, None) == -1
    assert gs(None, 2048, 64, None, 1, None, 8, 8, None, None, 1024, 8, 64, 2048, 1024, 3, None) == -1
    assert gs(None, 2048, 64, None, 1, None, 8, 8, None, None, 1024, 8, 64, 2048, 1000, 0, None) == -2
    assert lib.fnx_weighted_sum_f32(8, 8, 8, 0, 100, None) == -1                                 # no experts
    # the fused mix + router: decode shape rules and the decode workspace size; the flagged decode
    mr = lib.fnx_hc_mix_router
    assert mr(8, 8, 8, 8, 8, 1 << 30, 0, 2048, 512, 512, 10, 4, None) == -1                    # M = 0
    assert mr(8, 8, 8, 8, 8, 1 << 30, 1, 2000, 512, 512, 10, 4, None) == -2                    # H % 256
    assert mr(8, 8, 8, 8, 8, 16, 1, 2048, 512, 512, 10, 4, None) == -5                         # workspace
    assert lib.fnx_moe_decode_w4_ex(*([8] * 10), 1, 2048, 512, 512, 10, 8, 1 << 30, 2, None) == -1   # flags
    assert lib.fnx_weighted_sum_f32(None, 8, 8, 4, 100, None) == -1                              # no y
    assert lib.fnx_repack_w4_tiles(None, None, None, 8, 2048, 1024, 96, 0, None) == -1          # gs % 64
    assert lib.fnx_repack_v2o(None, 8, 1024, 2048, 0, None, None) == -1                          # no buffers
    assert lib.fnx_inject(None, None, None, None, 0, None) == -1                                  # batch 0
    assert lib.fnx_inject_ex(8, 8, 8, 8, 1, 100, 4, None) == -1                                   # H % 8
    assert lib.fnx_hc_activation(None, None, None, 0, 0, None) == -1                             # batch 0
    assert lib.fnx_hc_activation(8, 8, 8, 1, 4, None) == -1                                      # mode 4
    assert lib.fnx_hc_sigmoid_reduce_ex(8, 8, 8, 1, 2560, 0, None) == -1                         # HC 0
    assert lib.fnx_hc_rms_norm(8, 8, 8, 1, 0, 4, 1e-6, None) == -1                               # H 0
    ci = lib.fnx_moe_combine_inject
    assert ci(None, None, None, None, None, 1, 8, 8, 8, None, 4, 17, 2048, 4, None) == -1        # k > 16
    assert lib.fnx_repack_v2o(8, 8, 1024, 2000, 0, 8, None) == -1                                # K % 128
    assert lib.fnx_w4_tiles_bytes(512, 2048, 1024) == 512 * 8 * 32 * 4352
    assert lib.fnx_w4_tiles_bytes(512, 2048, 1000) == 0
    assert lib.fnx_w4gemv_launch(None, None, None, None, None, None, None, 1024, 100, 10, 20, 2, None) == -1
    assert lib.fnx_w4gemv_launch(None, None, None, None, None, None, None, 1024, 2048, 10, 20, 3, None) == -1
    assert lib.fnx_moe_decode_w4(*([None] * 10), 17, 2048, 512, 512, 10, None, 0, None) == -1
    assert lib.fnx_moe_decode_w4(*([None] * 10), 1, 2048, 512, 512, 10, None, 0, None) == -5
    # H or I of zero or below: rejected as shapes by all three decode entry points, and no
    # workspace size (a negative H would wrap the layout's offsets; I = 0 leaves groups that
    # never complete)
    for Hb, Ib in ((0, 512), (-256, 512), (2048, 0), (2048, -128), (128, 512), (2048, 64)):
        assert lib.fnx_moe_decode_w4(*([None] * 10), 1, Hb, Ib, 512, 10, None, 1 << 30, None) == -2, (Hb, Ib)
        assert lib.fnx_moe_decode_w4_noalloc(*([None] * 10), 1, Hb, Ib, 512, 10, None) == -2, (Hb, Ib)
        assert lib.fnx_moe_decode_workspace(1, Hb, Ib, 512, 10) == 0, (Hb, Ib)
    # W8A16: misaligned x / weights / scales / output are refused before either route (the GEMV
    # at M <= 16 and the tensor-core GEMM) launches
    w8 = lib.fnx_w8a16_gemm
    for M in (1, 300):
        assert w8(0x1008, 0x2000, 0x3000, 0x4000, M, 2048, 5120, 1, None) == -3, M     # x: 8 of 16 bytes
        assert w8(0x1000, 0x2004, 0x3000, 0x4000, M, 2048, 5120, 1, None) == -3, M     # w8t
        assert w8(0x1000, 0x2000, 0x3004, 0x4000, M, 2048, 5120, 1, None) == -3, M     # scales
        assert w8(0x1000, 0x2000, 0x3000, 0x4002, M, 2048, 5120, 1, None) == -3, M     # y
        assert lib.fnx_w8a16_gemm_ws(0x1000, 0x2000, 0x3000, 0x4002, M, 2048, 5120, 1, None, 0, None) == -3
    # expert-parallel dispatch layout and row gather
    d = lib.fnx_ep_dispatch_layout
    assert d(None, 40960, 512, 3, None, None, None, None, 0, None) == -1          # E % G
    assert d(None, 40960, 4, 8, None, None, None, None, 0, None) == -1            # G > E
    assert d(None, 40960, 512, 8, None, None, None, None, 0, None) == -1          # no counts
    assert d(None, 40960, 512, 8, None, None, 8, None, 0, None) == -5             # workspace
    gr = lib.fnx_ep_gather_rows
    assert gr(None, 2048, 10, None, 0, None, 1, None, 2048, None, 5, 2048, None) == -1      # index_div 0
    assert gr(None, 1000, 10, None, 1, None, 1, None, 2048, None, 5, 2048, None) == -1      # ld_src < H
    assert gr(None, 2048, 10, None, 1, None, 1, None, 2048, 8, 5, 2048, None) == -1         # ids_out w/o ids


def test_workspace_sizes(lib):
    assert lib.fnx_moe_permute_workspace(40960, 512) == 40 * 512 * 4
    assert lib.fnx_ep_layout_workspace(40960, 8) == 40 * 8 * 4 + 8 * 8
    assert lib.fnx_moe_decode_workspace(0, 2048, 512, 512, 10) == 0
    n1 = lib.fnx_moe_decode_workspace(1, 2048, 512, 512, 10)
    n16 = lib.fnx_moe_decode_workspace(16, 2048, 512, 512, 10)
    assert 0 < n1 < n16 < 64 << 20


def test_w8_split_workspace_sizes(lib):
    """The W8A16 split-K workspace: none where the GEMV serves (M <= 8) or where the GEMM has
    enough tiles (M = 200), s * M * N fp32 partials with s dividing K/64 in between, none for
    shapes the tensor-core GEMM does not take.  (Sizes only: nothing runs without a GPU; the
    split chosen assumes the 148 SMs of a B200 when no device is visible.)"""
    K, N = 2048, 5120
    assert lib.fnx_w8a16_gemm_workspace(8, K, N, 1) == 0
    assert lib.fnx_w8a16_gemm_workspace(200, K, N, 1) == 0
    for M in (9, 16, 64, 128):
        n = lib.fnx_w8a16_gemm_workspace(M, K, N, 1)
        s, rem = divmod(n, M * N * 4)
        assert rem == 0 and s > 1 and (K // 64) % s == 0 and s * M * 4 <= K, (M, n)
    assert lib.fnx_w8a16_gemm_workspace(16, K, 648, 1) == 0       # N % 128: the GEMV keeps M <= 16
    # splits that are not powers of two (K/64 = 24 or 48 k-blocks); the GPU tests run these cases
    for M, K2, s_want in ((12, 1536, 12), (64, 1536, 6), (100, 1536, 3), (64, 3072, 12)):
        n = lib.fnx_w8a16_gemm_workspace(M, K2, 640, 1)
        assert n == s_want * M * 640 * 4, (M, K2, n)
    assert lib.fnx_w8a16_gemm_workspace(16, K, N, 64) == 0        # 32-wide scale groups: GEMV as well


def test_python_wrappers_return_none_for_unsupported():
    import torch
    from fnx import expert_gather, moe_epilogue, post_ops, weighted_reduce
    v = torch.zeros(2, 10, 64, dtype=torch.bfloat16)
    assert weighted_reduce.reduce(v, torch.zeros(2, 10, dtype=torch.float32)) is None      # weights dtype
    assert weighted_reduce.reduce(v.view(20, 64), torch.zeros(2, 10, dtype=torch.bfloat16)) is None   # CPU tensors
    assert weighted_reduce.reduce(v, torch.zeros(2, 3, 64, dtype=torch.bfloat16), mean=True) is None
    assert post_ops.moe_merge(torch.zeros(1, 8, dtype=torch.bfloat16), torch.zeros(1, 8, dtype=torch.bfloat16),
                              torch.zeros(1, dtype=torch.bfloat16)) is None
    assert moe_epilogue.merge(torch.zeros(10, 640, dtype=torch.bfloat16), torch.zeros(1, 10, dtype=torch.bfloat16),
                              torch.zeros(1, 64, dtype=torch.bfloat16), torch.zeros(1, dtype=torch.bfloat16)) is None

    class P:
        expert_major = False
        _scales = None
    assert expert_gather.gather(P(), torch.zeros(10, dtype=torch.int64)) is None


def test_gated_residual_rejects_an_unsupported_fused_router():
    """gated_residual(..., moe=layer) refuses, before any launch, a batch or layer the fused mix +
    router kernel cannot take, instead of falling back to the unfused mix, after which the
    logits-ready decode the caller runs next would have no logits."""
    import torch
    from types import SimpleNamespace
    from fnx.engine import gated_residual
    H, hc = 256, 4
    w = torch.zeros(hc * H, dtype=torch.bfloat16)
    for b, moe in [(17, SimpleNamespace(E=64, H=H)), (2, SimpleNamespace(E=1024, H=H)),
                   (2, SimpleNamespace(E=64, H=2 * H))]:
        with pytest.raises(ValueError):
            gated_residual(torch.zeros(b, 1, hc * H, dtype=torch.bfloat16), w, None, None, moe=moe)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from fnx import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("FNX_B200_SO", str(tmp_path / "missing.so"))
    with pytest.raises(OSError):
        _lib.lib()


def test_expq_value_packer_matches_artifact(golden):
    """ExpQ(q, ...) turns int4 values into the LQP v2o bytes before the GPU repack: the
    packer reproduces the reference's artifact bytes from their unpacked values, and a
    CPU-resident ExpQ is refused (no CPU path)."""
    import torch
    import oracle as O
    from fnx.engine import ExpQ, _values_to_v2o
    g = golden("v2o")
    q = torch.from_numpy(O.unpack_v2o(g["v2o"].numpy(), g["K"])).to(torch.int8)
    assert torch.equal(_values_to_v2o(q), g["v2o"])
    with pytest.raises(RuntimeError):
        ExpQ(q, torch.ones(q.shape[0], q.shape[1], g["K"] // 64, dtype=torch.int8), 64)
