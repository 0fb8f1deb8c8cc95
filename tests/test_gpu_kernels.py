"""Per-kernel parity on the GPU: every C-ABI kernel against the CPU oracle.

Integer/index work (KV scatter, uniforms, slot FIFO, sampled token ids given the
same logits) must match bit for bit; floating-point kernels compare against the
oracle's fp32 math with the tolerance written in each test.
"""

from __future__ import annotations

import math

import pytest
import torch

from aios_b200 import _lib
from aios_b200.kernel import ops
from oracle import ops as oops
from oracle import sampler as osamp

pytestmark = pytest.mark.gpu


def _bf16_close(actual: torch.Tensor, expected: torch.Tensor, ulps: float = 2.0, atol: float = 1e-6) -> None:
    """|a - e| <= ulps * bf16 spacing(|e|) + atol, elementwise."""
    a, e = actual.float().cpu(), expected.float().cpu()
    spacing = torch.clamp(e.abs(), min=2.0**-126) * 2.0**-7
    bad = (a - e).abs() > ulps * spacing + atol
    assert not bool(bad.any()), f"{int(bad.sum())} mismatches; max abs diff {float((a - e).abs().max())}"


@pytest.mark.parametrize("rows", [1, 8, 13, 33, 100, 300, 700, 2048])
@pytest.mark.parametrize("n,k", [(1280, 768), (768, 768), (768, 2048), (1152, 768), (16384, 768)])
def test_linear_tcgen05_matches_fp32(cuda_device, rows: int, n: int, k: int) -> None:
    g = torch.Generator().manual_seed(rows * 7 + n + k)
    x = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    y = ops.linear(x.to(cuda_device), w.to(cuda_device))
    torch.cuda.synchronize()
    ops.check_status(cuda_device)
    # fp32 accumulation in a different order + one bf16 rounding: 1 ulp + tiny abs.
    _bf16_close(y, ref, ulps=1.0, atol=1e-4 * math.sqrt(k))


@pytest.mark.parametrize("rows", [1, 8, 33, 300, 2048])
def test_linear_silu_mul_epilogue(cuda_device, rows: int) -> None:
    g = torch.Generator().manual_seed(5 + rows)
    f, k = 2048, 768
    x = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * f, k, generator=g) * 0.02).to(torch.bfloat16)
    gate_up = (x.float() @ w.float().T).to(torch.bfloat16)  # reference rounds gate_up to bf16
    ref = oops.silu_and_mul(gate_up)
    y = ops.linear(x.to(cuda_device), ops.pack_gate_up(w.to(cuda_device)), epilogue=_lib.EPI_SILU_MUL)
    torch.cuda.synchronize()
    assert y.shape == (rows, f)
    _bf16_close(y, ref, ulps=2.0, atol=1e-4)


@pytest.mark.parametrize("rows", [8, 100, 2048])
@pytest.mark.parametrize("n,k", [(768, 768), (768, 2048)])
def test_linear_add_epilogue(cuda_device, rows: int, n: int, k: int) -> None:
    """y = residual + bf16(x W^T) (the o / down projections' residual add), with
    split-K reductions over clusters at every size."""
    g = torch.Generator().manual_seed(rows + n + k)
    x = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    res = torch.randn(rows, n, generator=g).to(torch.bfloat16)
    delta = (x.float() @ w.float().T).to(torch.bfloat16)
    ref = res.float() + delta.float()
    rd = res.to(cuda_device)
    y = ops.linear(x.to(cuda_device), w.to(cuda_device), out=rd, epilogue=_lib.EPI_ADD, residual=rd)
    torch.cuda.synchronize()
    ops.check_status(cuda_device)
    # the delta may differ from the fp32 reference's rounding by 1 ulp of itself
    spacing = torch.clamp(delta.float().abs(), min=2.0**-126) * 2.0**-7
    diff = (y.float().cpu() - ref).abs()
    assert bool((diff <= spacing + ref.abs() * 2.0**-8 + 1e-4 * math.sqrt(k)).all())


def test_rmsnorm_variants(cuda_device) -> None:
    g = torch.Generator().manual_seed(3)
    x = torch.randn(13, 768, generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(768, generator=g)).to(torch.bfloat16)
    y = ops.rmsnorm(x.to(cuda_device), w.to(cuda_device), 1e-6)
    _bf16_close(y, oops.rmsnorm(x, w, 1e-6), ulps=1.0)
    # per-head view of a packed qkv row: [T, H, d] with token stride > H*d
    qkv = torch.randn(5, 1280, generator=g).to(torch.bfloat16)
    hw = (1.0 + 0.1 * torch.randn(64, generator=g)).to(torch.bfloat16)
    qd = qkv.to(cuda_device)
    view = qd[:, :768].view(5, 12, 64)
    ops.rmsnorm(view, hw.to(cuda_device), 1e-6, out=view)
    ref = oops.rmsnorm(qkv[:, :768].view(5, 12, 64), hw, 1e-6)
    _bf16_close(qd[:, :768].view(5, 12, 64), ref, ulps=1.0)
    assert torch.equal(qd[:, 768:].cpu(), qkv[:, 768:])  # untouched k/v part


def test_fused_add_rmsnorm_and_silu(cuda_device) -> None:
    g = torch.Generator().manual_seed(4)
    x = torch.randn(9, 768, generator=g).to(torch.bfloat16)
    r = torch.randn(9, 768, generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(768, generator=g)).to(torch.bfloat16)
    xd, rd = x.to(cuda_device), r.to(cuda_device)
    ops.fused_add_rmsnorm(xd, rd, w.to(cuda_device), 1e-6)
    ex, er = oops.fused_add_rmsnorm(x, r, w, 1e-6)
    assert torch.equal(rd.cpu(), er)  # residual sum rounds once: bit-exact
    _bf16_close(xd, ex, ulps=1.0)
    gu = torch.randn(7, 4096, generator=g).to(torch.bfloat16)
    _bf16_close(ops.silu_and_mul(gu.to(cuda_device)), oops.silu_and_mul(gu), ulps=1.0)


def test_embedding_and_kv_store_bit_exact(cuda_device) -> None:
    g = torch.Generator().manual_seed(6)
    table = torch.randn(100, 768, generator=g).to(torch.bfloat16)
    ids = torch.tensor([5, 0, 99, 42], dtype=torch.int64)
    out = ops.embedding(ids.to(cuda_device), table.to(cuda_device))
    assert torch.equal(out.cpu(), table[ids])
    # store_cache into a [slots, Hkv, d] cache from strided k/v views of qkv
    slots, hkv, d = 64, 4, 64
    kc = torch.zeros(slots, hkv, d, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    qkv = torch.randn(6, 1280, generator=g).to(torch.bfloat16).to(cuda_device)
    k = qkv[:, 768:1024].view(6, hkv, d)
    v = qkv[:, 1024:].view(6, hkv, d)
    idx = torch.tensor([3, 60, 7, 0, 31, 12], dtype=torch.int32, device=cuda_device)
    ops.store_cache(kc, vc, idx, k, v)
    torch.cuda.synchronize()
    ops.check_status(cuda_device)
    assert torch.equal(kc[idx.long()].cpu(), k.cpu()) and torch.equal(vc[idx.long()].cpu(), v.cpu())
    untouched = torch.ones(slots, dtype=torch.bool)
    untouched[idx.long().cpu()] = False
    assert int(kc.cpu()[untouched].abs().sum()) == 0


@pytest.mark.parametrize("sources,tokens,partial", [(8, 8, True), (1, 8, True), (9, 8, False), (4, 33, True), (8, 4096, True),
                                                    (9, 5003, True), (1, 4096, False), (3, 9000, False)])
def test_attnres_mix_matches_oracle(cuda_device, sources: int, tokens: int, partial: bool) -> None:
    g = torch.Generator().manual_seed(11 + sources + tokens)
    bank = torch.randn(sources, tokens, 768, generator=g).to(torch.bfloat16)
    part = torch.randn(tokens, 768, generator=g).to(torch.bfloat16) if partial else None
    wq = torch.randn(768, generator=g) * 0.02
    out = ops.b200_attnres_mix(
        bank.to(cuda_device), None if part is None else part.to(cuda_device), wq.to(cuda_device), 1e-6
    )
    fused = oops.attnres_mix_fused(bank, part, wq, 1e-6)
    eager = oops.attnres_mix_eager(bank, part, wq, 1e-6)
    # the depth weights are rounded to bf16 (as the reference does); a score that
    # differs from the oracle's in its last fp32 bits can flip one weight's
    # rounding, which moves that token's outputs by up to one weight ulp (2^-8)
    # times the source value: every element within that, and at most 0.1% of the
    # elements beyond 1 ulp of the output
    src_max = float(bank.float().abs().max()) if part is None else max(float(bank.float().abs().max()),
                                                                      float(part.float().abs().max()))
    _bf16_close(out, fused, ulps=1.0, atol=2.0**-8 * src_max)
    a, e = out.float().cpu(), fused.float()
    over = (a - e).abs() > torch.clamp(e.abs(), min=2.0**-126) * 2.0**-7 + 1e-5
    assert float(over.float().mean()) <= 1e-3, f"{int(over.sum())} of {over.numel()} elements beyond 1 ulp"
    # the parity bar vs the eager (training) semantics: 1e-2 relative
    torch.testing.assert_close(out.float().cpu(), eager.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("sources,partial", [(1, False), (1, True), (5, True), (8, True), (9, False), (9, True)])
def test_attnres_stream_kernel_matches_register_kernel(cuda_device, sources: int, partial: bool) -> None:
    """From 2048 tokens the mixer streams tiles through shared memory; its
    outputs equal the small-count register kernel's bit for bit (the same
    arithmetic), checked on windows of 8 tokens mixed on their own."""
    tokens = 4099  # not a multiple of the 4-token tile
    g = torch.Generator().manual_seed(5 + sources)
    bank = torch.randn(sources, tokens, 768, generator=g).to(torch.bfloat16).to(cuda_device)
    part = torch.randn(tokens, 768, generator=g).to(torch.bfloat16).to(cuda_device) if partial else None
    wq = (torch.randn(768, generator=g) * 0.02).to(cuda_device)
    out = ops.b200_attnres_mix(bank, part, wq, 1e-6)
    for start in (0, 4, 1000, 2047, 4091):
        win = slice(start, start + 8)
        small = ops.b200_attnres_mix(bank[:, win].contiguous(), None if part is None else part[win].contiguous(),
                                     wq, 1e-6)
        assert torch.equal(out[win], small), f"window at {start}"
    assert not torch.isnan(out.float()).any()


@pytest.mark.parametrize("sources,tokens,partial", [(1, 8, False), (3, 8, True), (9, 8, True), (9, 1, False), (5, 17, True)])
def test_attnres_mix_rmsnorm_matches_mix_then_norm(cuda_device, sources: int, tokens: int, partial: bool) -> None:
    """The mixer with the consuming RMSNorm folded in equals the mixer followed by
    the RMSNorm kernel: the mixer arithmetic is shared, only the sum of squares is
    reduced in another order (1 bf16 ulp)."""
    g = torch.Generator().manual_seed(31 + sources + tokens)
    bank = torch.randn(sources, tokens, 768, generator=g).to(torch.bfloat16).to(cuda_device)
    part = torch.randn(tokens, 768, generator=g).to(torch.bfloat16).to(cuda_device) if partial else None
    wq = (torch.randn(768, generator=g) * 0.02).to(cuda_device)
    nw = (1.0 + 0.1 * torch.randn(768, generator=g)).to(torch.bfloat16).to(cuda_device)
    fused = ops.b200_attnres_mix_rmsnorm(bank, part, wq, 1e-6, nw, 1e-6)
    want = ops.rmsnorm(ops.b200_attnres_mix(bank, part, wq, 1e-6), nw, 1e-6)
    _bf16_close(fused, want, ulps=1.0)
    # stable bank sources read before the dependency wait: the same result, bit for bit
    for stable in (sources - 1, sources):
        early = ops.b200_attnres_mix_rmsnorm(bank, part, wq, 1e-6, nw, 1e-6, stable_sources=stable)
        assert torch.equal(early, fused)
    with pytest.raises(ValueError, match="stable_sources"):
        ops.b200_attnres_mix_rmsnorm(bank, part, wq, 1e-6, nw, 1e-6, stable_sources=sources + 1)


@pytest.mark.parametrize("sources,stable,tokens,partial,silu", [
    (1, 0, 8, False, False),   # block 0, first layer: the embedding just written
    (1, 1, 8, True, True),
    (4, 3, 8, False, False),   # a block's first layer: the newest source read late
    (4, 4, 8, True, False),
    (8, 8, 8, True, True),     # the last block
    (9, 8, 5, False, True),    # the final-mixer shape, ragged rows
    (3, 3, 1, True, False),
])
def test_linear_attnres_rmsnorm_matches_mix_then_linear(cuda_device, sources, stable, tokens, partial, silu) -> None:
    """The mixer and its RMSNorm built inside the decode linear equal the mixer
    kernel followed by the linear, to the rounding of the depth weights (their
    dot products and sums of squares are reduced in another order)."""
    g = torch.Generator().manual_seed(71 + sources * 8 + tokens + stable)
    dev = cuda_device
    bank = torch.randn(sources, tokens, 768, generator=g).to(torch.bfloat16).to(dev)
    part = torch.randn(tokens, 768, generator=g).to(torch.bfloat16).to(dev) if partial else None
    wq = (torch.randn(768, generator=g) * 0.05).to(dev)
    nw = (1.0 + 0.1 * torch.randn(768, generator=g)).to(torch.bfloat16).to(dev)
    n = 4096 if silu else 1280
    w = (torch.randn(n, 768, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    wk = ops.pack_gate_up(w) if silu else w
    epi = _lib.EPI_SILU_MUL if silu else _lib.EPI_STORE
    y = ops.linear_attnres_rmsnorm(bank, part, stable, wq, 1e-6, nw, 1e-6, wk, epilogue=epi)
    normed = ops.b200_attnres_mix_rmsnorm(bank, part, wq, 1e-6, nw, 1e-6)
    ref = ops.linear(normed, wk, epilogue=epi)
    torch.cuda.synchronize()
    ops.check_status(dev)
    _bf16_close(y, ref, ulps=3.0, atol=2e-3)
    with pytest.raises(ValueError):
        ops.linear_attnres_rmsnorm(bank, part, -1, wq, 1e-6, nw, 1e-6, wk, epilogue=epi)


def test_attnres_mix_rejects_bad_layout(cuda_device) -> None:
    bank = torch.zeros(2, 3, 768, dtype=torch.bfloat16, device=cuda_device)
    wq = torch.zeros(768, device=cuda_device)
    with pytest.raises(ValueError, match="partial must match"):
        ops.b200_attnres_mix(bank, torch.zeros(3, 767, dtype=torch.bfloat16, device=cuda_device), wq, 1e-6)
    with pytest.raises(ValueError, match="contiguous"):
        ops.b200_attnres_mix(bank.transpose(0, 1), None, wq, 1e-6)


def _rope_tables(d: int, max_pos: int, device):
    cos, sin = oops.rope_cache(d, max_pos, 1e6)
    return cos, sin, cos.to(torch.bfloat16).to(device), sin.to(torch.bfloat16).to(device)


STAGED, PREFIX_ONCE = _lib.HISTORY_STAGED, _lib.HISTORY_PREFIX_ONCE
DECODE_CASES = [
    # prefix, suffix (incl. the new token), page_size, history mode (0 = cascade
    # kernel, 1 = staged, 2 = prefix-once cluster staging), inactive rows, rows
    (13, 5, 1, 0, False, 8),
    (13, 5, 16, 0, False, 8),
    (13, 5, 1, STAGED, False, 8),
    (13, 5, 16, STAGED, False, 8),
    (13, 1, 1, STAGED, False, 8),    # first decode step: no older suffix keys
    (150, 40, 1, STAGED, True, 8),   # older suffix beyond the staged capacity
    (0, 9, 1, STAGED, False, 8),     # no shared prefix
    (150, 40, 1, 0, True, 8),
    (13, 5, 16, PREFIX_ONCE, False, 8),
    (13, 1, 1, PREFIX_ONCE, True, 8),
    (150, 40, 1, PREFIX_ONCE, True, 8),
    (0, 9, 1, PREFIX_ONCE, False, 8),
    (5, 3, 1, PREFIX_ONCE, False, 3),    # a 3-row cluster, slices of 1-2 prefix keys
    (37, 4, 16, PREFIX_ONCE, True, 13),  # clusters of 8 rows: 16 grid rows, 3 of them padding
    (440, 12, 16, STAGED, False, 8),     # a long prefix, staged whole (head_dim 64 and 96)
    (440, 12, 16, PREFIX_ONCE, False, 8),
    (500, 8, 1, PREFIX_ONCE, True, 8),   # beyond the head_dim-96 capacity: the rest streamed
]


def _decode_case(hq, hkv, d, prefix, suffix, page_size, inactive, rows, device):
    """Inputs of one decode-attention case and the oracle's output: `rows`
    candidate rows sharing a prefix, `suffix` own keys each (the newest one
    normalised, rotated and stored by the kernel)."""
    g = torch.Generator().manual_seed(hq * d + page_size + prefix + suffix + rows)
    num_pages = 64 if page_size == 16 else 1024
    if page_size == 16:
        num_pages = max(num_pages, (prefix + 15) // 16 + rows + 1)
    num_slots = num_pages * page_size
    width = 512 if prefix + suffix > 256 else 256
    cos, sin, cos_b, sin_b = _rope_tables(d, 512, device)
    eps, scale = 1e-6, d**-0.5
    kc = torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16)
    table = torch.zeros(rows, width, dtype=torch.int32)
    if page_size == 1:
        perm = torch.randperm(num_slots, generator=g)
        prefix_slots = perm[:prefix]
        suffix_slots = [perm[prefix + r * suffix : prefix + (r + 1) * suffix] for r in range(rows)]
    else:
        # the prefix on its own pages (the last one partly used), each row's suffix on its own page
        pages = torch.randperm(num_pages, generator=g)
        npp = (prefix + 15) // 16
        prefix_slots = (pages[:npp, None] * page_size + torch.arange(16)).flatten()[:prefix]
        suffix_slots = [pages[npp + r] * page_size + torch.arange(suffix) for r in range(rows)]
    for r in range(rows):
        table[r, :prefix] = prefix_slots.to(torch.int32)
        table[r, prefix : prefix + suffix] = suffix_slots[r].to(torch.int32)
    qkv = torch.randn(rows, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    qn = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    kn = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    pos = prefix + suffix - 1
    out_loc = table[:, pos].clone()
    active = torch.ones(rows, dtype=torch.int32)
    if inactive:
        active[[1, rows - 2]] = 0
    # oracle: norm + rope + store + attention
    q = qkv[:, : hq * d].view(rows, hq, d)
    k = qkv[:, hq * d : (hq + hkv) * d].view(rows, hkv, d)
    v = qkv[:, (hq + hkv) * d :].view(rows, hkv, d)
    qr = oops.apply_rope(oops.rmsnorm(q, qn, eps), cos[[pos] * rows], sin[[pos] * rows])
    kr = oops.apply_rope(oops.rmsnorm(k, kn, eps), cos[[pos] * rows], sin[[pos] * rows])
    kc_ref, vc_ref = kc.clone(), vc.clone()
    on = active.bool()
    kc_ref[out_loc[on].long()] = kr[on]
    vc_ref[out_loc[on].long()] = v[on]
    expected = torch.stack([
        oops.attention(qr[r : r + 1], kc_ref[table[r, : pos + 1].long()], vc_ref[table[r, : pos + 1].long()],
                       torch.tensor([pos]), scale)[0] if on[r] else torch.zeros(hq, d)
        for r in range(rows)
    ])
    dev = device
    args = dict(
        page_table=table.to(dev), row_table=torch.arange(rows, dtype=torch.int32, device=dev),
        seq_lens=torch.full((rows,), pos + 1, dtype=torch.int32, device=dev),
        positions=torch.full((rows,), pos, dtype=torch.int32, device=dev),
        num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, scale=scale,
        qkv=qkv.to(dev), q_norm_w=qn.to(dev), k_norm_w=kn.to(dev), eps=eps, cos=cos_b, sin=sin_b,
        out_loc=out_loc.to(dev), prefix_len=torch.tensor([prefix], dtype=torch.int32, device=dev),
        active=active.to(dev),
    )
    return kc, vc, kc_ref, vc_ref, expected, args


@pytest.mark.parametrize("hq,hkv,d", [(12, 4, 64), (8, 2, 96)])
@pytest.mark.parametrize("prefix,suffix,page_size,stable,inactive,rows", DECODE_CASES)
def test_cascade_decode_attention_fused_prologue(cuda_device, hq: int, hkv: int, d: int, prefix: int, suffix: int,
                                                 page_size: int, stable: int, inactive: bool, rows: int) -> None:
    """Candidate rows sharing a prefix, `suffix` own keys each (the newest one
    normalised, rotated and stored by the kernel itself); every kernel path."""
    kc, vc, kc_ref, vc_ref, expected, args = _decode_case(hq, hkv, d, prefix, suffix, page_size, inactive, rows,
                                                          cuda_device)
    dev = cuda_device
    kcd, vcd = kc.to(dev), vc.to(dev)
    out = torch.empty(rows, hq * d, dtype=torch.bfloat16, device=dev)
    # long prefixes staged whole (up to the head_dim's capacity); 150 keys with the
    # default 128-key staging, the rest read after the wait
    staged = prefix if prefix >= 256 else 0
    ops.attention_decode(out=out, k_cache=kcd, v_cache=vcd, stable_history=stable, staged_prefix=staged, **args)
    torch.cuda.synchronize()
    ops.check_status(dev)
    # the stored K must be the bf16 rope of the bf16 norm, bit for bit (active rows
    # only; an inactive row's slot keeps its old content)
    assert torch.equal(kcd.cpu(), kc_ref)
    assert torch.equal(vcd.cpu(), vc_ref)
    _bf16_close(out.view(rows, hq, d), expected, ulps=2.0, atol=2e-3)


@pytest.mark.parametrize("prefix,rows", [(13, 8), (77, 5), (440, 8), (300, 16)])
def test_prefix_once_staging_matches_per_row_staging(cuda_device, prefix: int, rows: int) -> None:
    """The prefix-once cluster staging and the per-row staging fold the same keys
    in the same order: outputs and stored K/V bit for bit."""
    hq, hkv, d = 12, 4, 64
    kc, vc, _, _, _, args = _decode_case(hq, hkv, d, prefix, 6, 16, True, rows, cuda_device)
    outs = []
    for mode in (STAGED, PREFIX_ONCE):
        kcd, vcd = kc.to(cuda_device), vc.to(cuda_device)
        out = torch.empty(rows, hq * d, dtype=torch.bfloat16, device=cuda_device)
        ops.attention_decode(out=out, k_cache=kcd, v_cache=vcd, stable_history=mode, staged_prefix=prefix, **args)
        torch.cuda.synchronize()
        ops.check_status(cuda_device)
        outs.append((out.cpu(), kcd.cpu(), vcd.cpu()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("stable", [0, 1, 2])
def test_decode_attention_reports_out_of_pool_slot(cuda_device, stable: int) -> None:
    """A page-table entry outside the KV pool is read as slot 0 (the kernel never
    indexes past the pool) and reported through the status word."""
    g = torch.Generator().manual_seed(11)
    rows, hq, hkv, d, prefix, suffix = 8, 12, 4, 64, 13, 5
    num_slots = 512
    cos, sin, cos_b, sin_b = _rope_tables(d, 512, cuda_device)
    perm = torch.randperm(num_slots, generator=g)
    table = torch.zeros(rows, 256, dtype=torch.int32)
    for r in range(rows):
        table[r, :prefix] = perm[:prefix].to(torch.int32)
        table[r, prefix : prefix + suffix] = perm[prefix + r * suffix : prefix + (r + 1) * suffix].to(torch.int32)
    pos = prefix + suffix - 1
    out_loc = table[:, pos].clone()
    table[3, prefix + 1] = num_slots + 7  # an older suffix key of row 3
    dev = cuda_device
    ops.check_status(dev)  # start from a clean status word
    out = torch.empty(rows, hq * d, dtype=torch.bfloat16, device=dev)
    ops.attention_decode(
        out=out, k_cache=torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16).to(dev),
        v_cache=torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16).to(dev), page_table=table.to(dev),
        row_table=torch.arange(rows, dtype=torch.int32, device=dev),
        seq_lens=torch.full((rows,), pos + 1, dtype=torch.int32, device=dev),
        positions=torch.full((rows,), pos, dtype=torch.int32, device=dev),
        num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, scale=d**-0.5,
        qkv=torch.randn(rows, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16).to(dev),
        q_norm_w=torch.ones(d, dtype=torch.bfloat16, device=dev), k_norm_w=torch.ones(d, dtype=torch.bfloat16, device=dev),
        eps=1e-6, cos=cos_b, sin=sin_b, out_loc=out_loc.to(dev),
        prefix_len=torch.tensor([prefix], dtype=torch.int32, device=dev),
        active=torch.ones(rows, dtype=torch.int32, device=dev), stable_history=stable,
    )
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="KV slot index outside the pool"):
        ops.check_status(dev)
    ops.check_status(dev)  # the status word was reset


@pytest.mark.parametrize("hq,hkv,d", [(12, 4, 64), (8, 2, 96)])
def test_prefill_attention_with_cached_prefix(cuda_device, hq: int, hkv: int, d: int) -> None:
    g = torch.Generator().manual_seed(21 + d)
    cached, new = 9, 24
    total = cached + new
    num_slots = 128
    cos, sin, cos_b, sin_b = _rope_tables(d, 512, cuda_device)
    eps, scale = 1e-6, d**-0.5
    perm = torch.randperm(num_slots, generator=g)
    slots = perm[:total].to(torch.int32)
    kc = torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16)
    qkv = torch.randn(new, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    qn = torch.ones(d, dtype=torch.bfloat16)
    kn = torch.ones(d, dtype=torch.bfloat16)
    positions = torch.arange(cached, total, dtype=torch.int32)
    q = qkv[:, : hq * d].view(new, hq, d)
    k = qkv[:, hq * d : (hq + hkv) * d].view(new, hkv, d)
    v = qkv[:, (hq + hkv) * d :].view(new, hkv, d)
    qr = oops.apply_rope(oops.rmsnorm(q, qn, eps), cos[positions.long()], sin[positions.long()])
    kr = oops.apply_rope(oops.rmsnorm(k, kn, eps), cos[positions.long()], sin[positions.long()])
    kc_ref, vc_ref = kc.clone(), vc.clone()
    kc_ref[slots[cached:].long()] = kr
    vc_ref[slots[cached:].long()] = v
    expected = oops.attention(qr, kc_ref[slots.long()], vc_ref[slots.long()], positions, scale)
    dev = cuda_device
    table = torch.zeros(1, 64, dtype=torch.int32)
    table[0, :total] = slots
    kcd, vcd = kc.to(dev), vc.to(dev)
    qbuf = torch.empty(new, hq * d, dtype=torch.bfloat16, device=dev)
    ops.qk_norm_rope_store(
        qkv=qkv.to(dev), num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, q_norm_w=qn.to(dev), k_norm_w=kn.to(dev),
        eps=eps, cos=cos_b, sin=sin_b, positions=positions.to(dev), out_loc=slots[cached:].to(dev),
        k_cache=kcd, v_cache=vcd, q_out=qbuf,
    )
    tile = ops.prefill_tile_tokens(hq, hkv)
    meta, ntiles = ops.prefill_meta([new], [cached], [0], tile)
    out = torch.empty(new, hq * d, dtype=torch.bfloat16, device=dev)
    ops.attention_prefill(
        q=qbuf, out=out, k_cache=kcd, v_cache=vcd, page_table=table.to(dev),
        meta=torch.tensor(meta, dtype=torch.int32, device=dev), num_requests=1, num_tiles=ntiles,
        tile_tokens=tile, num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, scale=scale,
    )
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert torch.equal(qbuf.cpu().view(new, hq, d), qr)
    assert torch.equal(kcd[slots[cached:].long()].cpu(), kr)
    _bf16_close(out.view(new, hq, d), expected, ulps=2.0, atol=2e-3)


@pytest.mark.parametrize("hq,hkv,d", [(12, 4, 64), (8, 2, 96), (16, 2, 128)])
def test_fused_prefill_matches_two_call_path(cuda_device, hq: int, hkv: int, d: int) -> None:
    """The one-launch prefill (norm, RoPE, K/V store, attention) against
    qk_norm_rope_store + attention_prefill, bit for bit, on a varlen batch: a
    fresh 13-token prefix, one token over 40 cached keys, and 64 new tokens over
    70 cached keys (chunks that mix cached and new keys)."""
    g = torch.Generator().manual_seed(5 + d)
    q_lens, cached_lens = [13, 1, 64], [0, 40, 70]
    num_slots, width = 1024, 256
    cos, sin, cos_b, sin_b = _rope_tables(d, 512, cuda_device)
    eps, scale = 1e-6, d**-0.5
    perm = torch.randperm(num_slots, generator=g)
    table = torch.zeros(len(q_lens), width, dtype=torch.int32)
    used = 0
    positions, out_loc = [], []
    for r, (n, c) in enumerate(zip(q_lens, cached_lens)):
        table[r, : c + n] = perm[used : used + c + n].to(torch.int32)
        used += c + n
        positions += list(range(c, c + n))
        out_loc += table[r, c : c + n].tolist()
    tokens = sum(q_lens)
    dev = cuda_device
    qkv = torch.randn(tokens, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16).to(dev)
    qn = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).to(dev)
    kn = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).to(dev)
    kc = torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    vc = torch.randn(num_slots, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    pos_d = torch.tensor(positions, dtype=torch.int32, device=dev)
    loc_d = torch.tensor(out_loc, dtype=torch.int32, device=dev)
    table_d = table.to(dev)
    tile = ops.prefill_tile_tokens(hq, hkv)
    meta_host, ntiles = ops.prefill_meta(q_lens, cached_lens, list(range(len(q_lens))), tile)
    meta = torch.tensor(meta_host, dtype=torch.int32, device=dev)

    kc_ref, vc_ref = kc.clone(), vc.clone()
    qbuf = torch.empty(tokens, hq * d, dtype=torch.bfloat16, device=dev)
    ops.qk_norm_rope_store(
        qkv=qkv, num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, q_norm_w=qn, k_norm_w=kn, eps=eps, cos=cos_b,
        sin=sin_b, positions=pos_d, out_loc=loc_d, k_cache=kc_ref, v_cache=vc_ref, q_out=qbuf,
    )
    expected = torch.empty(tokens, hq * d, dtype=torch.bfloat16, device=dev)
    ops.attention_prefill(
        q=qbuf, out=expected, k_cache=kc_ref, v_cache=vc_ref, page_table=table_d, meta=meta,
        num_requests=len(q_lens), num_tiles=ntiles, tile_tokens=tile, num_qo_heads=hq, num_kv_heads=hkv,
        head_dim=d, scale=scale,
    )
    out = torch.empty(tokens, hq * d, dtype=torch.bfloat16, device=dev)
    ops.attention_prefill_fused(
        qkv=qkv, out=out, q_norm_w=qn, k_norm_w=kn, eps=eps, cos=cos_b, sin=sin_b, positions=pos_d,
        out_loc=loc_d, k_cache=kc, v_cache=vc, page_table=table_d, meta=meta, num_requests=len(q_lens),
        num_tiles=ntiles, tile_tokens=tile, max_q_len=max(q_lens), num_qo_heads=hq, num_kv_heads=hkv,
        head_dim=d, scale=scale,
    )
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert torch.equal(out, expected)
    assert torch.equal(kc, kc_ref)
    assert torch.equal(vc, vc_ref)
    with pytest.raises(Exception, match="at most 64 new tokens"):
        ops.attention_prefill_fused(
            qkv=qkv, out=out, q_norm_w=qn, k_norm_w=kn, eps=eps, cos=cos_b, sin=sin_b, positions=pos_d,
            out_loc=loc_d, k_cache=kc, v_cache=vc, page_table=table_d, meta=meta, num_requests=len(q_lens),
            num_tiles=ntiles, tile_tokens=tile, max_q_len=65, num_qo_heads=hq, num_kv_heads=hkv,
            head_dim=d, scale=scale,
        )


@pytest.mark.parametrize("temperature,top_k,top_p", [(0.8, 50, 0.9), (0.75, 96, 0.95), (1.0, 1, 1.0), (0.35, 50, 1.0), (0.9, 0, 1.0)])
def test_sampler_tokens_bit_exact(cuda_device, temperature: float, top_k: int, top_p: float) -> None:
    g = torch.Generator().manual_seed(int(temperature * 100) + top_k)
    rows, vocab = 64, 16384
    logits = (torch.randn(rows, vocab, generator=g) * 2.0).to(torch.bfloat16)
    u = osamp.stateless_uniforms(list(range(1000, 1000 + rows)), 1)[:, 0]
    forbidden = [2, 3, 4]
    ban_rows = torch.randint(0, vocab, (rows, 3), generator=g)
    exp_tok, exp_lp = osamp.sample_with_logprobs(
        logits, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u,
        forbidden_token_ids=forbidden, forbidden_token_ids_by_row=ban_rows,
    )
    tok, lp = ops.sample(
        logits.to(cuda_device), temperature=temperature, top_k=top_k, top_p=top_p,
        greedy=osamp.is_greedy(temperature, top_k, top_p), uniforms=u.to(cuda_device),
        forbidden=torch.tensor(forbidden, dtype=torch.int32, device=cuda_device),
        forbidden_rows=ban_rows.to(cuda_device),
    )
    torch.cuda.synchronize()
    mism = (tok.cpu() != exp_tok).squeeze(-1)
    if bool(mism.any()):
        margins = osamp.sample_margin(logits, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u,
                                      forbidden_token_ids=forbidden, forbidden_token_ids_by_row=ban_rows)
        # a mismatch is only acceptable as a CDF-boundary rounding tie
        assert float(margins[mism.numpy()].max()) < 1e-6, f"token mismatch rows {mism.nonzero().flatten().tolist()}"
    torch.testing.assert_close(lp.cpu(), exp_lp, rtol=0, atol=2e-5)


# Every branch of the device sampler: the thread-maximum threshold path (k <= 512)
# and its fallbacks (k > 512: radix select; a row of ties: |C| > 2048), the full
# sort (top_k 0, top_p < 1), the sequential cumsum (probabilities below 2^-29),
# ragged and unaligned rows (scalar loads).
SAMPLER_PATHS = [
    ("k160", 16384, 0.75, 160, 0.95, "randn"),
    ("k512", 16384, 0.8, 512, 0.9, "randn"),
    ("k513_radix", 16384, 0.8, 513, 0.9, "randn"),
    ("k2048_radix", 16384, 1.0, 2048, 0.99, "randn"),
    ("ties_fallback", 16384, 0.8, 50, 0.9, "const"),
    ("few_distinct", 16384, 0.8, 50, 0.9, "coarse"),
    ("full_sort", 2048, 0.8, 0, 0.9, "randn"),
    # sorted sets above the 2048-entry top-k buffer sort whole rows in shared memory
    ("k4096_full_row", 16384, 0.8, 4096, 0.9, "randn"),
    ("k4096_no_topp", 16384, 1.0, 4096, 1.0, "randn"),
    ("topp_only_16384", 16384, 0.8, 0, 0.9, "randn"),
    ("topp_only_6401", 6401, 0.7, 0, 0.95, "randn"),
    # seven distinct values: the full sort orders ties by id (no top-p cut here,
    # which inside a tie group would depend on the last fp32 bits of the cumsum)
    ("topk_vocab_ties", 16384, 0.8, 16384, 1.0, "coarse"),
    ("tiny_probs", 16384, 0.5, 512, 1.0, "spread"),
    ("tiny_probs_topp", 16384, 0.5, 400, 0.999999, "spread"),
    ("s06_vocab", 6400, 0.8, 50, 0.9, "randn"),
    ("ragged_vocab", 6401, 0.8, 50, 0.9, "randn"),
    ("unaligned_row", 16384, 0.8, 50, 0.9, "unaligned"),
    ("greedy_unaligned", 6401, 1.0, 1, 1.0, "unaligned"),
    # the sorted paths rank unscaled logits unless a value could make two scaled
    # values collide: |v| near the fp32 limit for t < 2, t >= 2^16, -inf below t 2
    ("huge_fallback", 16384, 0.5, 50, 0.9, "huge"),
    ("high_temperature_fallback", 16384, 1e5, 50, 0.9, "randn"),
    ("neg_inf_fallback", 16384, 0.8, 50, 0.9, "neginf"),
    ("neg_inf_raw", 16384, 2.5, 50, 0.9, "neginf"),
]


@pytest.mark.parametrize("name,vocab,temperature,top_k,top_p,mode", SAMPLER_PATHS, ids=[c[0] for c in SAMPLER_PATHS])
def test_sampler_paths_bit_exact(cuda_device, name, vocab, temperature, top_k, top_p, mode) -> None:
    g = torch.Generator().manual_seed(len(name) * 7 + vocab)
    rows = 24
    if mode == "const":
        logits = torch.zeros(rows, vocab).to(torch.bfloat16)
    elif mode == "coarse":
        logits = torch.randint(-3, 4, (rows, vocab), generator=g).float().to(torch.bfloat16)
    elif mode == "spread":
        logits = (torch.randn(rows, vocab, generator=g) * 12.0).to(torch.bfloat16)
    elif mode in ("huge", "neginf"):
        logits = torch.randn(rows, vocab, generator=g) * 2.0
        idx = torch.randint(0, vocab, (rows, 6), generator=g)
        if mode == "huge":  # finite after scaling (|v| / t < 3.4e38), above the raw-key bound
            vals = torch.tensor([1e38, -1e38, 6e37, 9e37, -5e37, 1.2e38]).expand(rows, 6)
        else:
            vals = torch.full((rows, 6), float("-inf"))
        logits = logits.scatter(1, idx, vals).to(torch.bfloat16)
    else:
        logits = (torch.randn(rows, vocab, generator=g) * 2.0).to(torch.bfloat16)
    u = osamp.stateless_uniforms(list(range(77, 77 + rows)), 1)[:, 0]
    forbidden = [5, 6, 7, 100]
    ban_rows = torch.randint(0, vocab, (rows, 2), generator=g)
    exp_tok, exp_lp = osamp.sample_with_logprobs(
        logits, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u,
        forbidden_token_ids=forbidden, forbidden_token_ids_by_row=ban_rows,
    )
    if mode == "unaligned":
        wide = torch.zeros(rows, vocab + 1, dtype=torch.bfloat16)
        wide[:, 1:] = logits
        dev_logits = wide.to(cuda_device)[:, 1:]  # 2-byte offset rows: scalar loads
    else:
        dev_logits = logits.to(cuda_device)
    tok, lp = ops.sample(
        dev_logits, temperature=temperature, top_k=top_k, top_p=top_p,
        greedy=osamp.is_greedy(temperature, top_k, top_p), uniforms=u.to(cuda_device),
        forbidden=torch.tensor(forbidden, dtype=torch.int32, device=cuda_device),
        forbidden_rows=ban_rows.to(cuda_device),
    )
    torch.cuda.synchronize()
    ops.check_status(cuda_device)
    mism = (tok.cpu() != exp_tok).squeeze(-1)
    if bool(mism.any()):
        # a mismatch is only acceptable as a CDF-boundary rounding tie: the uniform
        # lies within 1e-6 of a boundary of the fp32 CDF, or (candidate sets of
        # thousands, where the fp32 softmax sum itself is off by a few 1e-6) within
        # the gap between the fp32 and the exact CDF
        bans = dict(forbidden_token_ids=forbidden, forbidden_token_ids_by_row=ban_rows)
        margins = osamp.sample_margin(logits, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u, **bans)
        band = osamp.cdf_rounding_band(logits, temperature=temperature, top_k=top_k, top_p=top_p, **bans)
        bad = (margins >= band + 1e-6) & mism.numpy()
        assert not bad.any(), f"{name}: token mismatch rows {bad.nonzero()[0].tolist()} " \
                              f"margins {margins[bad].tolist()} bands {band[bad].tolist()}"
    torch.testing.assert_close(lp.cpu(), exp_lp, rtol=0, atol=2e-5)


def test_stateless_uniforms_bit_exact(cuda_device) -> None:
    seeds = [20260814 + 100003 * 8 + i for i in range(8)] + [0, 1, 2**40 + 7]
    expected = osamp.stateless_uniforms(seeds, 16)
    got = ops.stateless_uniforms_device(torch.tensor(seeds, dtype=torch.int64, device=cuda_device), 16)
    assert torch.equal(got.cpu(), expected)


def test_slot_fifo_matches_reference_order(cuda_device) -> None:
    cap = 50
    ring = torch.arange(cap, dtype=torch.int32, device=cuda_device)
    model = list(range(cap))
    head, tail = 0, cap
    a = ops.slot_alloc(ring, head, 13)
    head += 13
    assert a.cpu().tolist() == model[:13]
    model = model[13:]
    ops.slot_free(ring, tail, a[5:9])
    tail += 4
    model += a[5:9].cpu().tolist()
    b = ops.slot_alloc(ring, head, 30)
    head += 30
    assert b.cpu().tolist() == model[:30]
    model = model[30:]
    # free b's range straight from the ring (overlapping wrap-around copy)
    ops.slot_free_range(ring, head - 30, 30, tail)
    tail += 30
    model += b.cpu().tolist()
    c = ops.slot_alloc(ring, head, tail - head)
    assert c.cpu().tolist() == model


@pytest.mark.parametrize("rows", [1, 8, 13, 33, 64])
@pytest.mark.parametrize("with_res,epi", [(True, "store"), (False, "store"), (True, "silu")])
def test_linear_with_fused_rmsnorm(cuda_device, rows: int, with_res: bool, epi: str) -> None:
    g = torch.Generator().manual_seed(50 + rows)
    k = 768
    n = 4096 if epi == "silu" else 1280
    x = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    r = torch.randn(rows, k, generator=g).to(torch.bfloat16) if with_res else None
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    if with_res:
        normed, new_res = oops.fused_add_rmsnorm(x, r, nw, 1e-6)
    else:
        normed, new_res = oops.rmsnorm(x, nw, 1e-6), None
    ref = normed.float() @ w.float().T
    dev = cuda_device
    res_out = torch.empty(rows, k, dtype=torch.bfloat16, device=dev) if with_res else None
    if epi == "silu":
        y = ops.linear_rmsnorm(x.to(dev), None if r is None else r.to(dev), nw.to(dev), 1e-6,
                               ops.pack_gate_up(w.to(dev)), residual_out=res_out, epilogue=_lib.EPI_SILU_MUL)
        ref = oops.silu_and_mul(ref.to(torch.bfloat16))
    else:
        y = ops.linear_rmsnorm(x.to(dev), None if r is None else r.to(dev), nw.to(dev), 1e-6, w.to(dev),
                               residual_out=res_out)
    torch.cuda.synchronize()
    ops.check_status(dev)
    # the normalised operand may differ from the oracle by one bf16 ulp (fp32 sum
    # order), so allow 2 ulps on the output
    _bf16_close(y, ref, ulps=2.0, atol=2e-3)
    if with_res:
        assert torch.equal(res_out.cpu(), new_res)


@pytest.mark.parametrize("rows", [1, 8, 13, 64, 100, 300, 700])
@pytest.mark.parametrize("epi", ["store", "silu"])
def test_residual_statistics_chain(cuda_device, rows: int, epi: str) -> None:
    """o_proj with the add+statistics epilogue, then a GEMM that normalises its
    input from those statistics: equals fused_add_rmsnorm followed by a linear."""
    g = torch.Generator().manual_seed(900 + rows)
    dev = cuda_device
    d, ka = 768, 768
    a = torch.randn(rows, ka, generator=g).to(torch.bfloat16)
    wo = (torch.randn(d, ka, generator=g) * 0.02).to(torch.bfloat16)
    res = torch.randn(rows, d, generator=g).to(torch.bfloat16)
    nw = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    n = 4096 if epi == "silu" else 1280
    w = (torch.randn(n, d, generator=g) * 0.02).to(torch.bfloat16)
    # reference: o = bf16(a Wo^T) from the same GEMM; fused_add_rmsnorm(o, res)
    o = ops.linear(a.to(dev), wo.to(dev)).cpu()
    normed, new_res = oops.fused_add_rmsnorm(o, res, nw, 1e-6)
    s_ref = o.float() + res.float()
    ref = normed.float() @ w.float().T
    res_dev = res.to(dev)
    stats = ops.linear_add_stat(a.to(dev), wo.to(dev), res_dev)
    if epi == "silu":
        y = ops.linear_stat_norm(stats, nw.to(dev), 1e-6, ops.pack_gate_up(w.to(dev)), epilogue=_lib.EPI_SILU_MUL)
        ref = oops.silu_and_mul(ref.to(torch.bfloat16))
    else:
        y = ops.linear_stat_norm(stats, nw.to(dev), 1e-6, w.to(dev))
    torch.cuda.synchronize()
    ops.check_status(dev)
    # the residual update is bit-exact (same GEMM, same rounding points)
    assert torch.equal(res_dev.cpu(), new_res)
    assert torch.equal(stats.x.cpu(), s_ref)
    # parts: 8-column groups (the register-operand path, up to 512 rows) or
    # 128-column tiles (tcgen05)
    assert stats.parts == (d // 8 if rows <= 512 else d // 128)
    part = (s_ref * s_ref).view(rows, stats.parts, d // stats.parts).sum(-1).T
    torch.testing.assert_close(stats.ss.cpu(), part, rtol=1e-5, atol=1e-5)
    _bf16_close(y, ref, ulps=2.0, atol=2e-3)


def _tile_stats_of(y: torch.Tensor) -> torch.Tensor:
    """[n / 16, rows, 4] (max, sum of exp(v - max), min, NaN flag) of y's 16-column tiles."""
    t = y.float().view(y.shape[0], -1, 16)
    mx = t.amax(-1)
    return torch.stack((mx, torch.exp(t - mx[..., None]).sum(-1), t.amin(-1), t.isnan().any(-1).float()),
                       -1).transpose(0, 1).contiguous()


@pytest.mark.parametrize("rows", [1, 8, 13, 16])
def test_lm_head_tile_statistics(cuda_device, rows: int) -> None:
    """The LM head's store epilogue with per-16-column tile statistics: the
    logits are bit-identical to the plain statistics linear, the tile max and
    min are exact, the sums of exponentials within fp32 rounding."""
    g = torch.Generator().manual_seed(40 + rows)
    dev = cuda_device
    d, vocab = 768, 6400
    x = torch.randn(rows, d, generator=g).to(torch.bfloat16)
    nw = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    w = (torch.randn(vocab, d, generator=g) * 0.05).to(torch.bfloat16)
    _, stats = ops.embedding_stat(torch.arange(rows, device=dev), x.to(dev))
    plain = ops.linear_stat_norm(stats, nw.to(dev), 1e-6, w.to(dev))
    tiles = torch.full((vocab // 16 * rows * 4,), float("nan"), device=dev)
    y = ops.linear_stat_norm(stats, nw.to(dev), 1e-6, w.to(dev), tile_stats=tiles)
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert torch.equal(y, plain)
    got = tiles.view(vocab // 16, rows, 4).cpu()
    want = _tile_stats_of(y.cpu())
    assert torch.equal(got[..., 0], want[..., 0]) and torch.equal(got[..., 2], want[..., 2])
    assert not got[..., 3].any()
    torch.testing.assert_close(got[..., 1], want[..., 1], rtol=2e-6, atol=0)
    assert ops.tile_stats_eligible(16, d, vocab) and not ops.tile_stats_eligible(17, d, vocab)
    if rows == 16:
        stats17 = ops.embedding_stat(torch.arange(17, device=dev) % rows, x.to(dev))[1]
        with pytest.raises(ValueError):
            ops.linear_stat_norm(stats17, nw.to(dev), 1e-6, w.to(dev), tile_stats=tiles)


@pytest.mark.parametrize("rows", [1, 8, 16])
def test_lm_head_tile_statistics_plain_operand(cuda_device, rows: int) -> None:
    """The same tile statistics from the plain linear (the LM head on rows the
    final RMSNorm already wrote, as the Block AttnRes trunk has them)."""
    g = torch.Generator().manual_seed(70 + rows)
    dev = cuda_device
    d, vocab = 768, 16384
    x = torch.randn(rows, d, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(vocab, d, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    plain = ops.linear(x, w)
    tiles = torch.full((vocab // 16 * rows * 4,), float("nan"), device=dev)
    y = ops.linear(x, w, tile_stats=tiles)
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert torch.equal(y, plain)
    got = tiles.view(vocab // 16, rows, 4).cpu()
    want = _tile_stats_of(y.cpu())
    assert torch.equal(got[..., 0], want[..., 0]) and torch.equal(got[..., 2], want[..., 2])
    assert not got[..., 3].any()
    torch.testing.assert_close(got[..., 1], want[..., 1], rtol=2e-6, atol=0)


def test_embedding_statistics(cuda_device) -> None:
    g = torch.Generator().manual_seed(5)
    w = torch.randn(1000, 768, generator=g).to(torch.bfloat16)
    ids = torch.tensor([3, 999, 0, 512, 3], dtype=torch.int64)
    out, st = ops.embedding_stat(ids.to(cuda_device), w.to(cuda_device))
    torch.cuda.synchronize()
    ops.check_status(cuda_device)
    assert torch.equal(out.cpu(), w[ids])
    assert torch.equal(st.x.cpu(), w[ids].float())
    torch.testing.assert_close(st.ss.cpu()[0], (w[ids].float() ** 2).sum(-1), rtol=1e-5, atol=1e-4)
    nw = torch.ones(768, dtype=torch.bfloat16)
    lin = (torch.randn(1280, 768, generator=g) * 0.02).to(torch.bfloat16)
    y = ops.linear_stat_norm(st, nw.to(cuda_device), 1e-6, lin.to(cuda_device))
    ref = oops.rmsnorm(w[ids], nw, 1e-6).float() @ lin.float().T
    _bf16_close(y, ref, ulps=2.0, atol=2e-3)
