"""Kernel-level parity on the GPU, through the C ABI: the tcgen05 linear kernel against a torch
fp32 reference of the same product (BF16 and TF32 operands, partial tiles, every epilogue), its
corrected form (FP16 + FP8 correction terms) against float64 with its FP8 companion output bit for
bit, the
flash-attention kernel against a float64 reference of the reference's masks, RMSNorm against the
oracle, and the reference's own padded-stride GEMM-seam test (core/gpu_test.zig:56-101)."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsfm_b200 as tb  # noqa: E402
from oracle import binding as ob  # noqa: E402

pytestmark = pytest.mark.gpu

BF16, F16, F32 = 2, 1, 0
TORCH16 = {"bf16": torch.bfloat16, "f16": torch.float16}
CODE16 = {torch.bfloat16: BF16, torch.float16: F16}


def dev():
    return torch.device("cuda:0")


def stream_ptr():
    return torch.cuda.current_stream().cuda_stream


def linear(x, w, bias, y, out_mode, act, M, N, K):
    tb.check(tb.lib.tsfm_kernel_linear(x.data_ptr(), CODE16.get(x.dtype, F32), w.data_ptr(), CODE16.get(w.dtype, F32),
                                       None if bias is None else bias.data_ptr(), y.data_ptr(), out_mode, act,
                                       M, N, K, x.stride(0), w.stride(0), y.stride(0), stream_ptr()))
    torch.cuda.synchronize()


# M >= 4096 with N > 128 runs on CTA pairs (2-SM MMA, 256-row tiles): full and partial row, column
# and K tiles.
SHAPES = [(128, 256, 64), (300, 336, 48), (1000, 768, 768), (257, 128, 3072), (7, 64, 200), (4096, 2304, 768),
          (4097, 600, 200), (8191, 768, 64), (4500, 1000, 1032)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("dtype", ["bf16", "f16", "tf32"])
def test_linear_matches_torch_fp32(M, N, K, dtype):
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N * 3 + K)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.05
    bias = torch.randn(N, generator=g)
    if dtype in TORCH16:
        xd, wd = x.to(dev(), TORCH16[dtype]), w.to(dev(), TORCH16[dtype])
    else:
        # TF32 operands: round to the 10-bit mantissa first so the product is exact in fp32
        xd = x.to(dev()).view(torch.int32).add(0x1000).bitwise_and(~0x1FFF).view(torch.float32)
        wd = w.to(dev()).view(torch.int32).add(0x1000).bitwise_and(~0x1FFF).view(torch.float32)
    ref = xd.double() @ wd.double().T + bias.to(dev()).double()
    tol = 2e-5 * K ** 0.5 * ref.abs().max().item() + 1e-5
    # f32 store with bias
    y = torch.full((M, N), float("nan"), device=dev())
    linear(xd, wd, bias.to(dev()), y, 1, 0, M, N, K)
    assert (y.double() - ref).abs().max().item() <= tol
    # relu + 16-bit store (in the operand type)
    if dtype in TORCH16:
        yb = torch.zeros((M, N), device=dev(), dtype=TORCH16[dtype])
        linear(xd, wd, bias.to(dev()), yb, 0, 1, M, N, K)
        assert (yb.double() - ref.clamp_min(0)).abs().max().item() <= tol + 2 ** -8 * ref.abs().max().item()
    # accumulate into an existing residual
    base = torch.randn(M, N, generator=g).to(dev())
    y2 = base.clone()
    linear(xd, wd, None, y2, 2, 0, M, N, K)
    ref2 = base.double() + xd.double() @ wd.double().T
    assert (y2.double() - ref2).abs().max().item() <= tol


@pytest.mark.parametrize("M", [300, 5000])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_linear_gated_pairs(M, dtype):
    # act 3: y[:, 128 t + c] = g * silu(u) with g, u = columns c and 128 + c of the product's
    # 256-column block t (single-CTA tiles at M = 300, CTA pairs at M = 5000).
    N, K = 768, 320
    g = torch.Generator(device="cpu").manual_seed(M + 11)
    x = torch.randn(M, K, generator=g).to(dev(), TORCH16[dtype])
    w = (torch.randn(N, K, generator=g) * 0.05).to(dev(), TORCH16[dtype])
    y = torch.full((M, N // 2), float("nan"), device=dev(), dtype=TORCH16[dtype])
    tb.check(tb.lib.tsfm_kernel_linear(x.data_ptr(), CODE16[x.dtype], w.data_ptr(), CODE16[w.dtype], None, y.data_ptr(),
                                       0, 3, M, N, K, K, K, N // 2, stream_ptr()))
    torch.cuda.synchronize()
    p = (x.double() @ w.double().T).view(M, N // 256, 2, 128)
    ref = (p[:, :, 0] * torch.nn.functional.silu(p[:, :, 1])).reshape(M, N // 2)
    tol = 2 ** -7 * ref.abs().max().item() + 1e-3
    assert (y.double() - ref).abs().max().item() <= tol


def test_linear_pairs_match_single_cta_tiles():
    # The same products with and without CTA pairs (a child process with TSFM_GEMM_PAIRS=0) agree to
    # within the FP32 accumulation tolerance.
    import os
    import subprocess
    import sys
    code = (
        "import sys, torch; sys.path[:0] = [%r, %r]; import tsfm_b200 as tb; "
        "g = torch.Generator().manual_seed(5); x = torch.randn(6000, 768, generator=g).half().cuda(); "
        "w = (torch.randn(2304, 768, generator=g) * 0.05).half().cuda(); y = torch.zeros(6000, 2304).cuda(); "
        "tb.check(tb.lib.tsfm_kernel_linear(x.data_ptr(), 1, w.data_ptr(), 1, None, y.data_ptr(), 1, 0, 6000, 2304, "
        "768, 768, 768, 2304, torch.cuda.current_stream().cuda_stream)); torch.cuda.synchronize(); "
        "torch.save(y.cpu(), sys.argv[1])"
    ) % (os.path.join(os.path.dirname(tb.__file__), ".."), os.path.join(os.path.dirname(tb.__file__), "..", ".."))
    outs = []
    for flag in ("1", "0"):
        path = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"tsfm_pairs_{flag}_{os.getpid()}.pt")
        env = dict(os.environ, TSFM_GEMM_PAIRS=flag)
        subprocess.run([sys.executable, "-c", code, path], env=env, check=True, timeout=300)
        outs.append(torch.load(path))
        os.remove(path)
    ref = outs[1].double()
    assert (outs[0].double() - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()


def test_linear_padded_output_stride_keeps_padding():
    M, N, K = 200, 96, 64
    x = torch.randn(M, K, device=dev()).to(torch.bfloat16)
    w = torch.randn(N, K, device=dev()).to(torch.bfloat16)
    y = torch.full((M, N + 40), -12345.0, device=dev())
    tb.check(tb.lib.tsfm_kernel_linear(x.data_ptr(), BF16, w.data_ptr(), BF16, None, y.data_ptr(), 1, 0, M, N, K,
                                       K, K, N + 40, stream_ptr()))
    torch.cuda.synchronize()
    assert torch.all(y[:, N:] == -12345.0)
    ref = x.double() @ w.double().T
    assert (y[:, :N].double() - ref).abs().max().item() < 1e-3


def attention_ref(q, k, v, kv, rel, n, heads, scale, mode):
    """float64 restatement of the reference masks (core/attn.zig:35-67 + T5 -floatMax addition)."""
    G = q.shape[0] // n
    out = torch.zeros(q.shape[0], heads * 64, dtype=torch.float64)
    qd, kd, vd = q.double().cpu(), k.double().cpu(), v.double().cpu()
    for g in range(G):
        valid = kv[g].bool() if kv is not None else torch.ones(n, dtype=torch.bool)
        for h in range(heads):
            sl = slice(h * 64, (h + 1) * 64)
            s = qd[g * n:(g + 1) * n, sl] @ kd[g * n:(g + 1) * n, sl].T * scale
            if rel is not None:
                i = torch.arange(n)
                s = s + rel[h][(i[None, :] - i[:, None]) + n - 1].double()
            i = torch.arange(n)
            if mode == 0:
                allowed = valid[None, :].expand(n, n).clone()
                if not valid.any():
                    allowed[:] = True
                    s = torch.zeros_like(s)
            elif mode == 1:
                allowed = (i[None, :] == i[:, None]) | (valid[None, :] & (i[None, :] <= i[:, None]))
            else:
                allowed = (i[None, :] == i[:, None]) | valid[None, :]
            s = s.masked_fill(~allowed, float("-inf"))
            p = torch.softmax(s, dim=1)
            out[g * n:(g + 1) * n, sl] = p @ vd[g * n:(g + 1) * n, sl]
    return out


@pytest.mark.parametrize("n,mode,with_rel", [(129, 0, True), (577, 0, False), (11, 0, True), (160, 1, False),
                                             (70, 2, False), (64, 1, False)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_attention_matches_float64_reference(n, mode, with_rel, dtype):
    heads, G = 3, 4
    g = torch.Generator().manual_seed(n + mode)
    ld = 3 * heads * 64 + 8
    qkv = (torch.randn(G * n, ld, generator=g) * 0.7).to(TORCH16[dtype]).to(dev())
    q, k, v = qkv[:, :heads * 64], qkv[:, heads * 64:2 * heads * 64], qkv[:, 2 * heads * 64:3 * heads * 64]
    kv = (torch.rand(G, n, generator=g) > 0.3).to(torch.uint8)
    kv[1, :] = 0  # a group with no valid key
    kv[2, :] = 1
    rel = torch.randn(heads, 2 * n - 1, generator=g) if with_rel else None
    o = torch.zeros(G * n, heads * 64, device=dev(), dtype=TORCH16[dtype])
    kvd = kv.to(dev())
    reld = rel.to(dev()) if rel is not None else None
    scale = 1.0 if mode == 0 else 0.125
    tb.check(tb.lib.tsfm_kernel_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, o.data_ptr(), heads * 64,
                                          kvd.data_ptr(), None if reld is None else reld.data_ptr(), G, heads, n,
                                          scale, mode, CODE16[TORCH16[dtype]], stream_ptr()))
    torch.cuda.synchronize()
    ref = attention_ref(q, k, v, kv, rel, n, heads, scale, mode)
    err = (o.double().cpu() - ref).abs().max().item()
    assert err < (3e-2 if dtype == "bf16" else 5e-3), err


@pytest.mark.parametrize("n,with_rel", [(1, False), (17, False), (128, False), (129, False), (132, False),
                                        (133, False), (256, False), (257, False), (640, False), (1100, False),
                                        (1, True), (17, True), (129, True), (130, True), (257, True), (512, True),
                                        (513, True)])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_attention_tcgen05_path_edges(n, with_rel, dtype):
    """The tcgen05 kernel (key-validity mask; relative-position bias up to n = 512, the mma.sync
    kernel beyond): one and two query tiles per CTA, partial key tiles, the K / V rings wrapping
    many times, a group without valid keys (uniform), a group whose first 300 keys are invalid
    (rows start with an empty max), and scores that grow by more than 2^8 per key tile so the lazy
    O / row-sum rescale runs on every tile. n = 128 k + 1 (129, 257) runs the key-tail instance
    (the last key in the softmax threads, the largest score of the growing group); 132 and 133
    the plain one."""
    heads, G = 2, 4
    gen = torch.Generator().manual_seed(1000 + n)
    ld = 3 * heads * 64
    qkv = torch.randn(G * n, ld, generator=gen) * 0.5
    u = torch.randn(64, generator=gen)
    u = u / u.norm()
    for h in range(heads):  # group 3: q along u, k growing along u with the key index
        rows = slice(3 * n, 4 * n)
        qkv[rows, h * 64:(h + 1) * 64] += 2.0 * u
        ramp = (0.05 * torch.arange(n, dtype=torch.float32))[:, None] * u[None, :]
        qkv[rows, heads * 64 + h * 64:heads * 64 + (h + 1) * 64] += ramp
    qkv = qkv.to(TORCH16[dtype]).to(dev())
    q, k, v = qkv[:, :heads * 64], qkv[:, heads * 64:2 * heads * 64], qkv[:, 2 * heads * 64:]
    kv = (torch.rand(G, n, generator=gen) > 0.3).to(torch.uint8)
    kv[1, :] = 0
    kv[2, :min(n, 300)] = 0
    if n > 300:
        kv[2, 300] = 1
    kv[3, :] = 1
    rel = torch.randn(heads, 2 * n - 1, generator=gen) * 2 if with_rel else None
    reld = rel.to(dev()) if with_rel else None
    o = torch.full((G * n, heads * 64), float("nan"), device=dev(), dtype=TORCH16[dtype])
    kvd = kv.to(dev())
    tb.check(tb.lib.tsfm_kernel_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, o.data_ptr(), heads * 64,
                                          kvd.data_ptr(), None if reld is None else reld.data_ptr(), G, heads,
                                          n, 1.0, 0, CODE16[TORCH16[dtype]], stream_ptr()))
    torch.cuda.synchronize()
    ref = attention_ref(q, k, v, kv, rel, n, heads, 1.0, 0)
    got = o.double().cpu()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err < (3e-2 if dtype == "bf16" else 5e-3), err


@pytest.mark.parametrize("n,with_rel", [(1, False), (129, False), (256, False), (577, False), (1100, False),
                                        (17, True), (129, True), (257, True)])
@pytest.mark.parametrize("o8", [False, True])
def test_attention_split_rows(n, with_rel, o8):
    """The tcgen05 kernel with two softmax threads per query row (force_path 3): the groups of the
    edge test (uniform, leading invalid keys, scores growing past the rescale threshold on every
    tile), against float64, with and without the FP8 companion output."""
    from helpers import e4m3_bits
    heads, G = 2, 4
    gen = torch.Generator().manual_seed(2000 + n)
    ld = 3 * heads * 64
    qkv = torch.randn(G * n, ld, generator=gen) * 0.5
    u = torch.randn(64, generator=gen)
    u = u / u.norm()
    for h in range(heads):
        rows = slice(3 * n, 4 * n)
        qkv[rows, h * 64:(h + 1) * 64] += 2.0 * u
        ramp = (0.05 * torch.arange(n, dtype=torch.float32))[:, None] * u[None, :]
        qkv[rows, heads * 64 + h * 64:heads * 64 + (h + 1) * 64] += ramp
    qkv = qkv.half().to(dev())
    q, k, v = qkv[:, :heads * 64], qkv[:, heads * 64:2 * heads * 64], qkv[:, 2 * heads * 64:]
    kv = (torch.rand(G, n, generator=gen) > 0.3).to(torch.uint8)
    kv[1, :] = 0
    kv[2, :min(n, 300)] = 0
    if n > 300:
        kv[2, 300] = 1
    kv[3, :] = 1
    rel = torch.randn(heads, 2 * n - 1, generator=gen) * 2 if with_rel else None
    reld = rel.to(dev()) if with_rel else None
    kvd = kv.to(dev())
    width = heads * 64
    o = torch.full((G * n, width), float("nan"), device=dev(), dtype=torch.float16)
    o8b = torch.zeros(G * n, 2 * width, device=dev(), dtype=torch.uint8) if o8 else None
    tb.check(tb.lib.tsfm_kernel_attention_ex(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, o.data_ptr(), width, None, 0,
        o8b.data_ptr() if o8 else None, 2 * width, kvd.data_ptr(), n, None if reld is None else reld.data_ptr(),
        None, G, heads, n, 1.0, 0, n, n, F16, 3, stream_ptr()))
    torch.cuda.synchronize()
    got = o.double().cpu()
    assert torch.isfinite(got).all()
    ref = attention_ref(q, k, v, kv, rel, n, heads, 1.0, 0)
    assert (got - ref).abs().max().item() < 5e-3
    if o8:
        xh = o.float().cpu().numpy()
        assert np.array_equal(o8b.cpu().numpy()[:, :width], e4m3_bits(xh * np.float32(1 / 32)))


def timestral_attention_ref(q, k, v, kv, bidir, n, heads, scale, ne, l):
    """float64 restatement of Timestral's time-attention masks (timestral/model.zig:558-635):
    encoder queries i < ne see j < ne with j == i or (valid(j) and (bidirectional or j <= i));
    decoder queries i >= ne see valid j < l plus ne <= j <= i."""
    G = q.shape[0] // n
    out = torch.zeros(q.shape[0], heads * 64, dtype=torch.float64)
    qd, kd, vd = q.double().cpu(), k.double().cpu(), v.double().cpu()
    i = torch.arange(n)[:, None]
    j = torch.arange(n)[None, :]
    for g in range(G):
        valid = kv[g].bool()[None, :]
        bd = bool(bidir[g])
        enc = (j < ne) & ((j == i) | (valid & (bd | (j <= i))))
        dec = ((j < l) & valid) | ((j >= ne) & (j <= i))
        allowed = torch.where(i < ne, enc, dec)
        for h in range(heads):
            sl = slice(h * 64, (h + 1) * 64)
            s = qd[g * n:(g + 1) * n, sl] @ kd[g * n:(g + 1) * n, sl].T * scale
            p = torch.softmax(s.masked_fill(~allowed, float("-inf")), dim=1)
            out[g * n:(g + 1) * n, sl] = p @ vd[g * n:(g + 1) * n, sl]
    return out


@pytest.mark.parametrize("n,ne,l,mode", [(160, 144, 128, 1), (160, 160, 160, 1), (17, 12, 8, 1), (129, 100, 64, 1),
                                         (300, 256, 200, 1), (700, 600, 512, 1), (200, 150, 150, 2), (1, 1, 1, 1),
                                         (256, 128, 0, 1)])
@pytest.mark.parametrize("out32", [False, True])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_attention_timestral_masks_both_paths(n, ne, l, mode, out32, dtype):
    """Timestral's causal / bidirectional / decoder-chain masks on the tcgen05 kernel (force_path 1,
    and 3: two softmax threads per row) and the mma.sync kernel (force_path 2), 16-bit and FP32
    outputs, against float64: groups with per-group bidirectional rows, invalid keys everywhere but
    the diagonal, and decoder rows."""
    heads, G = 2, 5
    gen = torch.Generator().manual_seed(7 * n + ne + l + mode)
    ld = 3 * heads * 64 + 8
    qkv = (torch.randn(G * n, ld, generator=gen) * 0.7).to(TORCH16[dtype]).to(dev())
    q, k, v = qkv[:, :heads * 64], qkv[:, heads * 64:2 * heads * 64], qkv[:, 2 * heads * 64:3 * heads * 64]
    kv = (torch.rand(G, ne, generator=gen) > 0.3).to(torch.uint8)
    kv[1, :] = 0  # only the diagonal (and the decoder chain) visible
    kv[2, :] = 1
    bidir = torch.tensor([0, 1, 0, 1, 0], dtype=torch.uint8)
    if mode == 2:
        bidir[:] = 1
    kv_full = torch.ones(G, n, dtype=torch.uint8)
    kv_full[:, :ne] = kv
    scale = 0.125
    ref = timestral_attention_ref(q, k, v, kv_full, bidir, n, heads, scale, ne, l)
    kvd, bidird = kv.to(dev()), bidir.to(dev())  # kept alive until the kernels have run
    outs = {}
    for path in (1, 2, 3):
        o = torch.full((G * n, heads * 64), float("nan"), device=dev(), dtype=TORCH16[dtype])
        o32 = torch.full((G * n, heads * 64), float("nan"), device=dev(), dtype=torch.float32) if out32 else None
        tb.check(tb.lib.tsfm_kernel_attention_ex(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, None if out32 else o.data_ptr(), heads * 64,
            o32.data_ptr() if out32 else None, heads * 64, None, 0, kvd.data_ptr(), ne, None,
            bidird.data_ptr(), G, heads, n, scale, mode, ne, l, CODE16[TORCH16[dtype]], path, stream_ptr()))
        torch.cuda.synchronize()
        outs[path] = (o32 if out32 else o).double().cpu()
        assert torch.isfinite(outs[path]).all(), path
        err = (outs[path] - ref).abs().max().item()
        assert err < (3e-2 if dtype == "bf16" else 5e-3), (path, err)
    if out32:
        assert (outs[1] - outs[2]).abs().max().item() < (3e-2 if dtype == "bf16" else 5e-3)


@pytest.mark.parametrize("n,pad8", [(1, 0), (129, 0), (577, 0), (129, 16)])
def test_attention_fp8_companion(n, pad8):
    """The tcgen05 kernel's FP8 companion of its FP16 output (corrected products), bit for bit:
    with x the kernel's FP32 output (the same launch with an FP32 output), the FP16 output is
    f16(x) and the companion [e4m3(f16(x) / 32) | e4m3((x - f16(x)) * 128)]. pad8 = 16: a
    companion row stride that is 16- but not 32-byte aligned (16-byte stores instead of 32-byte
    ones); the padding bytes stay untouched."""
    from helpers import e4m3_bits
    heads, G = 2, 3
    gen = torch.Generator().manual_seed(77 + n)
    ld = 3 * heads * 64
    qkv = (torch.randn(G * n, ld, generator=gen) * 0.7).half().to(dev())
    q, k, v = qkv[:, :heads * 64], qkv[:, heads * 64:2 * heads * 64], qkv[:, 2 * heads * 64:]
    kv = (torch.rand(G, n, generator=gen) > 0.2).to(torch.uint8)
    kv[:, 0] = 1
    kvd = kv.to(dev())
    width = heads * 64
    o = torch.empty(G * n, width, device=dev(), dtype=torch.float16)
    o8 = torch.full((G * n, 2 * width + pad8), 0xA5, device=dev(), dtype=torch.uint8)
    o32 = torch.empty(G * n, width, device=dev(), dtype=torch.float32)
    for out, out32, out8 in ((o, None, o8), (None, o32, None)):
        tb.check(tb.lib.tsfm_kernel_attention_ex(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, None if out is None else out.data_ptr(), width,
            None if out32 is None else out32.data_ptr(), width, None if out8 is None else out8.data_ptr(),
            2 * width + pad8, kvd.data_ptr(), n, None, None, G, heads, n, 0.125, 0, n, n, F16, 1, stream_ptr()))
    torch.cuda.synchronize()
    x = o32.cpu().numpy()
    xh = x.astype(np.float16).astype(np.float32)
    assert np.array_equal(o.float().cpu().numpy(), xh)
    b8 = o8.cpu().numpy()
    assert (b8[:, 2 * width:] == 0xA5).all()
    b8 = b8[:, :2 * width]
    assert np.array_equal(b8[:, :width], e4m3_bits(xh * np.float32(1 / 32)))
    assert np.array_equal(b8[:, width:], e4m3_bits((x - xh) * np.float32(128)))
    ref = attention_ref(q, k, v, kv, None, n, heads, 0.125, 0).numpy()
    assert np.max(np.abs(x - ref)) < 5e-3


def test_rmsnorm_matches_oracle():
    rows, dim = 1000, 768
    rng = np.random.default_rng(1)
    x = rng.standard_normal((rows, dim)).astype(np.float32) * 3
    s = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    want = np.zeros_like(x)
    ob.lib.oracle_rmsnorm(x.ctypes.data, s.ctypes.data, want.ctypes.data, rows, dim, 1e-6)
    xd, sd = torch.from_numpy(x).to(dev()), torch.from_numpy(s).to(dev())
    out = torch.zeros(rows, dim, device=dev())
    tb.check(tb.lib.tsfm_kernel_rmsnorm(xd.data_ptr(), sd.data_ptr(), out.data_ptr(), F32, rows, dim, 1e-6,
                                        stream_ptr()))
    outb = torch.zeros(rows, dim, device=dev(), dtype=torch.bfloat16)
    tb.check(tb.lib.tsfm_kernel_rmsnorm(xd.data_ptr(), sd.data_ptr(), outb.data_ptr(), BF16, rows, dim, 1e-6,
                                        stream_ptr()))
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(outb.float().cpu().numpy(), want, rtol=2 ** -7, atol=1e-2)


@pytest.mark.parametrize("dim,pad8", [(256, 0), (768, 0), (768, 8), (1024, 0), (772, 0), (772, 8)])
def test_rmsnorm_fp8_companion(dim, pad8):
    """RMSNorm with the FP8 companion of its FP16 output (the corrected mode's norm), on both
    kernels: rows of 256 * k values take the 256-bit-access kernel, others (772) the general one.
    With y the same launch's FP32 output: FP16 output f16(y), companion [e4m3(f16(y) / 32) |
    e4m3((y - f16(y)) * 128)] bit for bit, y against the oracle. pad8: companion rows longer than
    2 * dim whose padding stays untouched."""
    from helpers import e4m3_bits
    rows = 1000
    rng = np.random.default_rng(dim + pad8)
    x = (rng.standard_normal((rows, dim)) * 3).astype(np.float32)
    s = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    xd, sd = torch.from_numpy(x).to(dev()), torch.from_numpy(s).to(dev())
    y = torch.zeros(rows, dim, device=dev())
    h = torch.zeros(rows, dim, device=dev(), dtype=torch.float16)
    b8 = torch.full((rows, 2 * dim + pad8), 0xA5, device=dev(), dtype=torch.uint8)
    tb.check(tb.lib.tsfm_kernel_rmsnorm_ex(xd.data_ptr(), sd.data_ptr(), y.data_ptr(), F32, None, 0, rows, dim, 1e-6,
                                           stream_ptr()))
    tb.check(tb.lib.tsfm_kernel_rmsnorm_ex(xd.data_ptr(), sd.data_ptr(), h.data_ptr(), F16, b8.data_ptr(),
                                           2 * dim + pad8, rows, dim, 1e-6, stream_ptr()))
    torch.cuda.synchronize()
    want = np.zeros_like(x)
    ob.lib.oracle_rmsnorm(x.ctypes.data, s.ctypes.data, want.ctypes.data, rows, dim, 1e-6)
    yv = y.cpu().numpy()
    np.testing.assert_allclose(yv, want, rtol=1e-5, atol=1e-5)
    yh = yv.astype(np.float16).astype(np.float32)
    assert np.array_equal(h.float().cpu().numpy(), yh)
    bb = b8.cpu().numpy()
    assert (bb[:, 2 * dim:] == 0xA5).all()
    assert np.array_equal(bb[:, :dim], e4m3_bits(yh * np.float32(1 / 32)))
    assert np.array_equal(bb[:, dim:2 * dim], e4m3_bits((yv - yh) * np.float32(128)))


def test_gemm_seam_padded_strides_like_reference_gpu_test():
    # core/gpu_test.zig:56-101: m, n, k = 37, 29, 23; lda, ldb, ldc = 31, 41, 47; sentinel -12345
    # must survive in the padding; tolerance 1e-4; registered-weight NT and activation NN paths.
    m, n, k, lda, ldb, ldc = 37, 29, 23, 31, 41, 47
    rng = np.random.default_rng(0x5EED)
    a = (rng.random(lda * m, dtype=np.float32) * 2 - 1)
    bnt = (rng.random(ldb * n, dtype=np.float32) * 2 - 1)
    bnn = (rng.random(ldb * k, dtype=np.float32) * 2 - 1)
    A = a.reshape(m, lda)[:, :k].astype(np.float64)
    BNT = bnt.reshape(n, ldb)[:, :k].astype(np.float64)
    BNN = bnn.reshape(k, ldb)[:, :n].astype(np.float64)
    out = np.full(ldc * m, -12345.0, np.float32)
    assert tb.lib.tsfm_sgemm_nt(m, n, k, 0.7, a.ctypes.data, lda, bnt.ctypes.data, ldb, out.ctypes.data, ldc, None) == 0
    o = out.reshape(m, ldc)
    np.testing.assert_allclose(o[:, :n], 0.7 * A @ BNT.T, atol=1e-4)
    assert np.all(o[:, n:] == -12345.0)
    wd = np.ascontiguousarray(BNT.astype(np.float32))
    h = tb.lib.tsfm_weight_register(wd.ctypes.data, wd.size)
    assert h
    out[:] = -12345.0
    assert tb.lib.tsfm_sgemm_nt(m, n, k, 0.7, a.ctypes.data, lda, wd.ctypes.data, k, out.ctypes.data, ldc, h) == 0
    np.testing.assert_allclose(o[:, :n], 0.7 * A @ BNT.T, atol=1e-4)
    assert np.all(o[:, n:] == -12345.0)
    tb.lib.tsfm_weight_release(h)
    out[:] = -12345.0
    assert tb.lib.tsfm_sgemm_nn(m, n, k, a.ctypes.data, lda, bnn.ctypes.data, ldb, out.ctypes.data, ldc, None) == 0
    np.testing.assert_allclose(o[:, :n], A @ BNN, atol=1e-4)
    assert np.all(o[:, n:] == -12345.0)
    # Registered weights read in place on the device with their padded row strides: NT over
    # [n, ldb] rows and NN over [k, ldb] rows (transposed on the device, never copied back).
    for kind, buf, want in (("nt", bnt, 0.7 * A @ BNT.T), ("nn", bnn, A @ BNN)):
        h = tb.lib.tsfm_weight_register(buf.ctypes.data, buf.size)
        assert h
        out[:] = -12345.0
        if kind == "nt":
            st = tb.lib.tsfm_sgemm_nt(m, n, k, 0.7, a.ctypes.data, lda, None, ldb, out.ctypes.data, ldc, h)
        else:
            st = tb.lib.tsfm_sgemm_nn(m, n, k, a.ctypes.data, lda, None, ldb, out.ctypes.data, ldc, h)
        tb.lib.tsfm_weight_release(h)
        assert st == 0, tb.last_error()
        np.testing.assert_allclose(o[:, :n], want, atol=1e-4)
        assert np.all(o[:, n:] == -12345.0)


# Corrected products (TSFM_COMPUTE_F16C): FP16 operands plus the FP8 first-order correction terms.
CORR_SHAPES = [(300, 336, 48), (1000, 768, 768), (257, 128, 3072), (4096, 2304, 768), (4500, 1000, 1032),
               (7, 64, 200)]


def linear_corrected(x, w, bias, y, y8, out_mode, act, terms=2):
    M, K = x.shape
    N = w.shape[0]
    tb.check(tb.lib.tsfm_kernel_linear_corrected(x.data_ptr(), w.data_ptr(), None if bias is None else bias.data_ptr(),
                                                 y.data_ptr(), None if y8 is None else y8.data_ptr(), out_mode, act,
                                                 M, N, K, terms, stream_ptr()))
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,N,K", CORR_SHAPES)
def test_linear_corrected_matches_float64(M, N, K):
    # The corrected product of FP32 x and W against float64: every element within 2^-12 of
    # sum_k |x_k w_k| (twice the first-order bound; a single FP16 product is off by up to 2^-10), and the RMS error at
    # least 8x below that of the plain FP16 product of the same operands.
    g = torch.Generator(device="cpu").manual_seed(M * 5 + N + K)
    x = torch.randn(M, K, generator=g).to(dev())
    w = (torch.randn(N, K, generator=g) * 0.05).to(dev())
    bias = torch.randn(N, generator=g).to(dev())
    ref = x.double() @ w.double().T + bias.double()
    mag = x.double().abs() @ w.double().abs().T + bias.double().abs()
    y = torch.full((M, N), float("nan"), device=dev())
    linear_corrected(x, w, bias, y, None, 1, 0)
    err = (y.double() - ref).abs()
    assert (err <= 2.0 ** -12 * mag + 1e-6).all()
    y16 = torch.full((M, N), float("nan"), device=dev())
    linear(x.half(), w.half(), bias, y16, 1, 0, M, N, K)
    rms = lambda t: t.pow(2).mean().sqrt().item()  # noqa: E731
    assert rms(err) * 8 <= rms(y16.double() - ref)
    # accumulate mode
    base = torch.randn(M, N, generator=g).to(dev())
    y2 = base.clone()
    linear_corrected(x, w, None, y2, None, 2, 0)
    assert ((y2.double() - base.double() - (ref - bias.double())).abs() <= 2.0 ** -12 * mag + 1e-5).all()


@pytest.mark.parametrize("M,N,K", [(300, 320, 48), (4096, 2304, 768), (257, 128, 3072)])
def test_linear_corrected_fp8_companion_bits(M, N, K):
    # A 16-bit output with its FP8 companion: y16 = f16(y) and the companion's bytes are exactly
    # e4m3(y16 / 32) and e4m3((y - y16) * 128), with y the same product stored in f32.
    from helpers import e4m3_bits
    g = torch.Generator(device="cpu").manual_seed(M + N + K + 1)
    x = torch.randn(M, K, generator=g).to(dev())
    w = (torch.randn(N, K, generator=g) * 0.05).to(dev())
    bias = torch.randn(N, generator=g).to(dev())
    y32 = torch.zeros((M, N), device=dev())
    linear_corrected(x, w, bias, y32, None, 1, 1)
    y16 = torch.zeros((M, N), device=dev(), dtype=torch.float16)
    y8 = torch.zeros((M, 2 * N), device=dev(), dtype=torch.uint8)
    linear_corrected(x, w, bias, y16, y8, 0, 1)
    a32, a16, a8 = y32.cpu().numpy(), y16.cpu().numpy(), y8.cpu().numpy()
    assert np.array_equal(a16.view(np.uint16), a32.astype(np.float16).view(np.uint16))
    h = a16.astype(np.float32)
    assert np.array_equal(a8[:, :N], e4m3_bits(h * np.float32(1 / 32)))
    assert np.array_equal(a8[:, N:], e4m3_bits((a32 - h) * np.float32(128)))


@pytest.mark.parametrize("M,N,K", [(300, 336, 48), (4096, 2304, 768), (257, 128, 3072)])
def test_linear_weight_term_only(M, N, K):
    # terms = 1: only x_hi (W - f16(W)) is added, so the result is the product of the FP16-rounded
    # input with the full-precision weight: against float64 of (f16(x), W), within 2^-12 of
    # sum_k |x_k w_k|.
    g = torch.Generator(device="cpu").manual_seed(M + 3 * N + K)
    x = torch.randn(M, K, generator=g).to(dev())
    w = (torch.randn(N, K, generator=g) * 0.05).to(dev())
    y = torch.full((M, N), float("nan"), device=dev())
    linear_corrected(x, w, None, y, None, 1, 0, terms=1)
    xh = x.half().double()
    ref = xh @ w.double().T
    mag = xh.abs() @ w.double().abs().T
    assert ((y.double() - ref).abs() <= 2.0 ** -12 * mag + 1e-6).all()
