"""Kernel-level parity on the GPU: each sm_100a kernel against the reference's own outputs
(tests/golden/*.npz) or, for floating-point contractions, an fp64 truth with a stated tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.harness import golden
from tests.streams import FILTER_CASES, STATS_CASES, filter_inputs, stats_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _kn():
    from proteus_b200 import kernels
    return kernels


@pytest.mark.parametrize("case", range(len(FILTER_CASES)))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_filter_matches_reference(case, dtype):
    """Survivor set, values and count of filter_candidates (filter_triton.py:65-86) — bit-exact,
    including the exact count when the output buffer overflows (cap 64)."""
    KN = _kn()
    H, rowmap, tp, tn = filter_inputs(case)
    Hd = torch.from_numpy(H).to(DEV).to(dtype)
    rm = torch.from_numpy(rowmap).to(DEV)
    tpd, tnd = torch.from_numpy(tp).to(DEV), torch.from_numpy(tn).to(DEV)
    v, r, c, cnt = KN.filter_candidates(Hd, rm, tpd, tnd, 1 << 16)
    n = int(cnt)
    if dtype == torch.bfloat16:  # the golden is the reference kernel on these bf16 inputs
        z = golden("filter")
        assert n == int(z[f"f{case}_count"])
        o = np.lexsort((c[:n].cpu().numpy(), r[:n].cpu().numpy()))
        assert np.array_equal(r[:n].cpu().numpy()[o], z[f"f{case}_row"])
        assert np.array_equal(c[:n].cpu().numpy()[o], z[f"f{case}_col"])
        assert np.array_equal(v[:n].cpu().numpy()[o], z[f"f{case}_val"])
    Hf = H.astype(np.float32)
    want = ((Hf > tp) | (-Hf > tn)) & (rowmap >= 0)[:, None]
    assert n == int(want.sum())
    _, _, _, cnt64 = KN.filter_candidates(Hd, rm, tpd, tnd, 64)
    assert int(cnt64) == n  # overflow: exact count, nothing past cap


@pytest.mark.parametrize("T,D", [(4099, 5120), (1031, 10240)])
def test_filter_large_vector_path(T, D):
    """bf16 16-byte vector path at B200-sized shapes (ESM-2 650M and 3B FFN widths) with a padding
    mix and -inf thresholds."""
    KN = _kn()
    g = torch.Generator(device=DEV).manual_seed(0)
    H = (torch.randn(T, D, generator=g, device=DEV) * 2).to(torch.bfloat16)
    valid = torch.rand(T, generator=g, device=DEV) > 0.1
    rowmap = torch.full((T,), -1, dtype=torch.int64, device=DEV)
    rowmap[valid] = torch.arange(int(valid.sum()), device=DEV)
    tp = torch.rand(D, generator=g, device=DEV) + 5.0
    tn = torch.rand(D, generator=g, device=DEV) + 5.0
    tn[:3] = float("-inf")
    v, r, c, cnt = KN.filter_candidates(H, rowmap, tp, tn, 1 << 20)
    n = int(cnt)
    Hf = H.float()
    mask = ((Hf > tp) | (-Hf > tn)) & valid[:, None]
    rt, ct = torch.nonzero(mask, as_tuple=True)
    assert n == rt.numel()
    got = torch.stack([r[:n], c[:n]], 1)
    want = torch.stack([rowmap[rt], ct], 1)
    key = lambda x: (x[:, 0] * D + x[:, 1]).sort().values  # noqa: E731
    assert torch.equal(key(got), key(want))
    inv = torch.nonzero(valid).squeeze(1)
    assert torch.equal(v[:n], Hf[inv[r[:n]], c[:n]])


def test_filter_density_mix_partial_strip():
    """TMA-fed bf16 path: ragged T, a partial last strip (D = 1000 = 3 x 256 + 232 columns), padding
    rows, and columns from near-dense (most values survive: more flagged rows per warp step than the
    hit queue holds) to sparse, against the fp32 comparison; plus the exact count past a small cap."""
    KN = _kn()
    g = torch.Generator(device=DEV).manual_seed(11)
    T, D = 1333, 1000
    H = torch.randn(T, D, generator=g, device=DEV).to(torch.bfloat16)
    valid = torch.rand(T, generator=g, device=DEV) > 0.07
    rowmap = torch.full((T,), -1, dtype=torch.int64, device=DEV)
    rowmap[valid] = torch.arange(int(valid.sum()), device=DEV)
    level = torch.rand(D, generator=g, device=DEV)
    tp = torch.where(level < 0.1, torch.full_like(level, -2.0), 1.5 + 2.0 * level)  # 10% near-dense columns
    tn = torch.where(level > 0.95, torch.full_like(level, -2.0), 1.5 + 2.0 * (1 - level))
    v, r, c, cnt = KN.filter_candidates(H, rowmap, tp, tn, 1 << 21)
    n = int(cnt)
    Hf = H.float()
    mask = ((Hf > tp) | (-Hf > tn)) & valid[:, None]
    rt, ct = torch.nonzero(mask, as_tuple=True)
    assert n == rt.numel()
    key = lambda a, b: (a * D + b).sort().values  # noqa: E731
    assert torch.equal(key(r[:n], c[:n]), key(rowmap[rt], ct))
    inv = torch.nonzero(valid).squeeze(1)
    assert torch.equal(v[:n], Hf[inv[r[:n]], c[:n]])
    _, _, _, cnt_small = KN.filter_candidates(H, rowmap, tp, tn, 1000)
    assert int(cnt_small) == n


def test_filter_bf16_threshold_edges():
    """bf16 path compares packed bf16 pairs against bf16-rounded thresholds; the survivors must be
    those of the fp32 comparison for thresholds equal to a bf16 value (ties do not survive),
    one fp32 ulp either side of it, +-inf, beyond the bf16 range, and NaN inputs/thresholds."""
    KN = _kn()
    g = torch.Generator(device=DEV).manual_seed(5)
    T, D = 1536, 1024
    H = (torch.randn(T, D, generator=g, device=DEV) * 3).to(torch.bfloat16)
    H[7, :64] = float("nan")
    H[9, 64:128] = float("inf")
    H[11, 128:192] = float("-inf")
    H[13, 192:256] = -0.0
    Hf = H.float()
    base = Hf[torch.randint(0, T, (D,), generator=g, device=DEV), torch.arange(D, device=DEV)].abs()
    tp, tn = base.clone(), base.clone()
    kind = torch.arange(D, device=DEV) % 8
    up = lambda x: torch.nextafter(x, torch.full_like(x, float("inf")))  # noqa: E731
    dn = lambda x: torch.nextafter(x, torch.full_like(x, float("-inf")))  # noqa: E731
    tp = torch.where(kind == 1, up(tp), tp)
    tp = torch.where(kind == 2, dn(tp), tp)
    tn = torch.where(kind == 3, up(tn), tn)
    tn = torch.where(kind == 4, dn(tn), tn)
    tp = torch.where(kind == 5, torch.full_like(tp, 3.395e38), tp)  # above the largest bf16
    tn = torch.where(kind == 5, torch.full_like(tn, float("inf")), tn)
    tn = torch.where(kind == 6, torch.full_like(tn, float("-inf")), tn)
    tp = torch.where(kind == 7, torch.full_like(tp, float("-inf")), tp)
    tp[0::97] = 0.0
    tn[1::89] = -0.0
    rowmap = torch.arange(T, dtype=torch.int64, device=DEV)
    rowmap[3::5] = -1
    v, r, c, cnt = KN.filter_candidates(H, rowmap, tp, tn, 1 << 22)
    n = int(cnt)
    valid = rowmap >= 0
    mask = ((Hf > tp) | (-Hf > tn)) & valid[:, None]
    rt, ct = torch.nonzero(mask, as_tuple=True)
    assert n == rt.numel()
    key = lambda a, b: (a * D + b).sort().values  # noqa: E731
    assert torch.equal(key(r[:n], c[:n]), key(rowmap[rt], ct))


@pytest.mark.parametrize("case", range(len(STATS_CASES)))
def test_sub_stats_matches_reference(case):
    """Bin masses and int8 masks bit-exact vs the reference kernel; sums within rtol 1e-5 (the
    reference test's tolerance, tests/test_stats_triton.py:45-46)."""
    KN = _kn()
    X, E0, E1, levels = stats_inputs(case)
    s, sq, cnt, M = KN.sub_stats(torch.from_numpy(X).to(DEV).to(torch.bfloat16), torch.from_numpy(E0).to(DEV),
                                 torch.from_numpy(E1).to(DEV), levels)
    z = golden("sub_stats")
    if f"s{case}_cnt" in z:
        assert np.array_equal(cnt.cpu().numpy(), z[f"s{case}_cnt"])
        assert np.array_equal(M.cpu().numpy(), z[f"s{case}_M"])
        assert np.allclose(s.cpu().numpy(), z[f"s{case}_sum"], rtol=1e-5, atol=1e-4)
        assert np.allclose(sq.cpu().numpy(), z[f"s{case}_sq"], rtol=1e-5, atol=1e-4)
    Xd = X.astype(np.float64)  # fp32 within 8-row groups, fp64 across: error far below 1e-6 of sum|x|
    assert (np.abs(s.cpu().numpy() - Xd.sum(0)) <= 1e-6 * np.abs(Xd).sum(0) + 1e-12).all()
    assert (np.abs(sq.cpu().numpy() - (Xd ** 2).sum(0)) <= 1e-6 * (Xd ** 2).sum(0) + 1e-12).all()


def test_sub_stats_bf16_edge_ties():
    """bf16 statistics compare packed pairs against edges rounded to bf16; counts and masks must be
    those of the fp32 compares for edges equal to values present in X (ties count: x >= E0,
    -x >= E1), one fp32 ulp either side, and +-0 / +-inf / NaN rows; a ragged n and mask padding."""
    KN = _kn()
    g = torch.Generator().manual_seed(9)
    n, D, B = 1001, 136, 5
    X = (torch.randn(n, D, generator=g) * 2).to(torch.bfloat16)
    X[3, :8] = float("nan")
    X[5, 8:16] = float("inf")
    X[6, 16:24] = float("-inf")
    X[7, 24:32] = -0.0
    X[8, 24:32] = 0.0
    Xf = X.float()
    pick = lambda: Xf[torch.randint(0, n, (D,), generator=g), torch.arange(D)].nan_to_num(0.0, 0.0, 0.0)  # noqa: E731
    E0 = torch.stack([pick() for _ in range(B)], 1).sort(1).values
    E1 = torch.stack([-pick() for _ in range(B)], 1).sort(1).values
    up = lambda x: torch.nextafter(x, torch.full_like(x, float("inf")))  # noqa: E731
    dn = lambda x: torch.nextafter(x, torch.full_like(x, float("-inf")))  # noqa: E731
    E0[1::3, 1], E0[2::3, 3] = up(E0[1::3, 1]), dn(E0[2::3, 3])
    E1[0::3, 2], E1[2::3, 4] = up(E1[0::3, 2]), dn(E1[2::3, 4])
    E0[:, 0] = torch.where(torch.arange(D) % 5 == 0, torch.zeros(D), E0[:, 0])
    E0, E1 = E0.sort(1).values.contiguous(), E1.sort(1).values.contiguous()
    levels = (2, 3, 4)
    s, sq, cnt, M = KN.sub_stats(X.to(DEV), E0.to(DEV), E1.to(DEV), levels)
    ge0 = Xf[:, :, None] >= E0[None]  # [n, D, B]
    ge1 = (-Xf)[:, :, None] >= E1[None]
    cum0, cum1 = ge0.sum(0), ge1.sum(0)  # [D, B]
    nxt = lambda c: torch.cat([c[:, 1:], torch.zeros(D, 1, dtype=c.dtype)], 1)  # noqa: E731
    want_cnt = torch.stack([cum0 - nxt(cum0), cum1 - nxt(cum1)]).to(torch.int32)
    assert torch.equal(cnt.cpu(), want_cnt)
    n8 = -(-n // 8) * 8
    for j, lv in enumerate(levels):
        m0 = torch.zeros(D, n8, dtype=torch.int8)
        m1 = torch.zeros(D, n8, dtype=torch.int8)
        m0[:, :n] = ge0[:, :, lv].T.to(torch.int8)
        m1[:, :n] = ge1[:, :, lv].T.to(torch.int8)
        assert torch.equal(M[0, j].cpu(), m0), j
        assert torch.equal(M[1, j].cpu(), m1), j


@pytest.mark.parametrize("n,D", [(1600, 5120), (301, 1000), (77, 96), (4096, 640), (700, 3900), (300, 10240)])
def test_gram_upper_blocks(n, D):
    """gram_accumulate semantics: two accumulations, rel-max error < 1e-5 vs fp64 (reference
    test tolerance, tests/test_stats_triton.py:74), lower 128-blocks untouched."""
    KN = _kn()
    g = torch.Generator().manual_seed(1)
    X1 = torch.randn(n, D, generator=g).to(torch.bfloat16)
    X2 = torch.randn(n // 2 + 3, D, generator=g).to(torch.bfloat16)
    C = torch.zeros(D, D, device=DEV)
    KN.gram_accumulate(X1.to(DEV), C)
    KN.gram_accumulate(X2.to(DEV), C)
    from proteus_b200.core import symmetrize_upper
    G = symmetrize_upper(C.cpu().double())
    R = X1.double().T @ X1.double() + X2.double().T @ X2.double()
    rel = float((G - R).abs().max() / R.abs().max())
    assert rel < 1e-5, rel
    nb = -(-D // 128)
    Cc = C.cpu()
    for i in range(nb):
        for j in range(i):
            assert bool((Cc[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128] == 0).all())


@pytest.mark.parametrize("M,n,A", [(30720 // 8, 1664, 21), (768, 128, 16), (384, 2048, 48)])
def test_count_gemm_i8_exact(M, n, A):
    KN = _kn()
    g = torch.Generator().manual_seed(2)
    masks = (torch.rand(M, n, generator=g) < 0.3).to(torch.int8)
    A_pad = max(16, -(-A // 16) * 16)
    annT = torch.zeros(A_pad, n, dtype=torch.int8)
    annT[:A] = (torch.rand(A, n, generator=g) < 0.2).to(torch.int8)
    out = torch.full((M, A), 7, dtype=torch.int64, device=DEV)
    KN.count_gemm_i8(masks.to(DEV), annT.to(DEV), out, A)
    want = masks.long() @ annT[:A].long().T + 7
    assert torch.equal(out.cpu(), want)


def test_grouped_merge_matches_reference():
    KN = _kn()
    z = golden("grouped_merge")
    I64_MIN = torch.iinfo(torch.int64).min
    for case in range(3):
        G, K, rounds = (int(x) for x in z[f"c{case}_meta"])
        st = torch.full((G, K), I64_MIN, dtype=torch.long, device=DEV)
        pt = torch.full((G, K), -1, dtype=torch.long, device=DEV)
        pv = torch.full((G, K), float("-inf"), device=DEV)
        for r in range(rounds):
            t = lambda k: torch.from_numpy(z[f"c{case}_r{r}_{k}"]).to(DEV)  # noqa: E731
            KN.grouped_merge(st, [pt, pv], t("g"), t("s"), [t("t"), t("v")], K)
        assert np.array_equal(st.cpu().numpy(), z[f"c{case}_state"])
        assert np.array_equal(pt.cpu().numpy(), z[f"c{case}_tok"])
        assert np.array_equal(pv.cpu().numpy(), z[f"c{case}_val"])


def test_grouped_merge_large_random_vs_oracle():
    """Many candidates per group (several 32-wide chunks), K=100, against the oracle's merge."""
    from oracle import atlas_np as O
    KN = _kn()
    rng = np.random.default_rng(3)
    G, K = 500, 100
    st = np.full((G, K), O.I64_MIN, np.int64)
    pt = np.full((G, K), -1, np.int64)
    pv = np.full((G, K), -np.inf, np.float32)
    dst = torch.from_numpy(st).to(DEV)
    dpt = torch.from_numpy(pt).to(DEV)
    dpv = torch.from_numpy(pv).to(DEV)
    for rnd in range(4):
        n = 40000
        g = rng.integers(0, G, n)
        sc = rng.choice(2**50, n, replace=False).astype(np.int64) - 2**49
        tok = rng.integers(0, 2**32, n)
        val = rng.standard_normal(n).astype(np.float32)
        O.grouped_merge(st, [pt, pv], g, sc, [tok, val], K, pay_fill=[-1, -np.inf])
        KN.grouped_merge(dst, [dpt, dpv], torch.from_numpy(g).to(DEV), torch.from_numpy(sc).to(DEV),
                         [torch.from_numpy(tok).to(DEV), torch.from_numpy(val).to(DEV)], K)
    assert np.array_equal(dst.cpu().numpy(), st)
    assert np.array_equal(dpt.cpu().numpy(), pt)
    assert np.array_equal(dpv.cpu().numpy(), pv)


def test_device_status_clean_after_tensor_core_kernels():
    """No bounded wait of the tcgen05 kernels gave up during this session."""
    import ctypes
    from proteus_b200 import _lib
    torch.cuda.synchronize()
    st = ctypes.c_int(-1)
    assert _lib.load().atlas_device_status(ctypes.byref(st), 0) == 0
    assert st.value == 0


# ----------------------------------------------------------------------------------------- pilot
def test_device_pilot_matches_reference_goldens():
    """The device pilot (atlas_column_select / _pilot_edges / _pilot_counts / _pilot_seeds) on the
    reference's pilot inputs (fp32; the second layer rounded to quarters, so edges fall on ties and
    on signed zeros) equals the reference's pilot_edges / pilot_seeds, with and without protein
    groups. Edges compare as floats (-0.0 == +0.0: the reference's own sort orders signed zeros
    arbitrarily, and no bin or threshold can tell them apart); seeds and key ceilings bit for bit."""
    from proteus_b200.pilot import pilot_edges, pilot_seeds
    from tests.streams import pilot_inputs
    Hs, groups = pilot_inputs()
    z = golden("pilot")
    Ht = [torch.from_numpy(h).to(DEV) for h in Hs]
    E = pilot_edges(Ht)
    assert E.is_cuda and np.array_equal(E.cpu().numpy(), z["E"])
    ts, rk = pilot_seeds(Ht, E, 16, 8, n_total=10**6, groups=torch.from_numpy(groups))
    assert np.array_equal(ts.numpy(), z["top_seed"]) and np.array_equal(rk.numpy(), z["res_seed_key"])
    ts0, rk0 = pilot_seeds(Ht, E, 16, 8, n_total=10**6)
    assert np.array_equal(ts0.numpy(), z["top_seed_nogroups"]) and np.array_equal(rk0.numpy(), z["res_seed_key_nogroups"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_device_pilot_matches_oracle_wide_shuffled_groups(dtype):
    """A wider pilot (n = 20011 rows, D = 1280) in bf16 / fp16 with proteins of random sizes whose
    ids are not sorted and whose rows are not contiguous: every edge, seed and key ceiling equals the
    oracle's (pinned to the reference) on the same values."""
    from oracle import atlas_np as O
    from proteus_b200.pilot import pilot_edges, pilot_seeds
    rng = np.random.default_rng(31)
    n, D = 20011, 1280
    H = (rng.standard_t(3, (n, D)) * (rng.random(D) + 0.5) + rng.standard_normal(D) * 0.5).astype(np.float32)
    Hd = torch.from_numpy(H).to(DEV).to(dtype)
    Hn = Hd.float().cpu().numpy()
    sizes = rng.integers(1, 400, 200)
    prot = np.repeat(rng.permutation(10**6)[:200], sizes)[:n]
    prot = np.concatenate([prot, np.full(n - prot.size, 77)])[rng.permutation(n)]
    E = pilot_edges([Hd])
    Eo = O.pilot_edges([Hn])
    assert np.array_equal(E.cpu().numpy(), Eo)
    ts, rk = pilot_seeds([Hd], E, 100, 32, n_total=190_000_000, groups=torch.from_numpy(prot))
    tso, rko = O.pilot_seeds([Hn], Eo, 100, 32, n_total=190_000_000, groups=prot)
    assert np.array_equal(ts.numpy(), tso) and np.array_equal(rk.numpy(), rko)
    ts0, rk0 = pilot_seeds([Hd], E, 100, 32, n_total=190_000_000)
    tso0, rko0 = O.pilot_seeds([Hn], Eo, 100, 32, n_total=190_000_000)
    assert np.array_equal(ts0.numpy(), tso0) and np.array_equal(rk0.numpy(), rko0)


# ----------------------------------------------------------------------------------------- fused stats + enrichment
@pytest.mark.parametrize("D,n,A,NL,col0", [(1333, 1611, 21, 3, 64), (5120, 16384, 32, 3, 0), (300, 300, 7, 2, 8),
                                           (257, 129, 48, 1, 0), (640, 9000, 16, 3, 24)])
def test_stats_enrich_fused_equals_two_kernel_path(D, n, A, NL, col0):
    """atlas_sub_stats_enrich (masks built in shared memory, int8 tcgen05 contraction) against
    atlas_sub_stats (masks written to HBM) + atlas_count_gemm_i8 on the same staged rows: bin masses
    and contingencies bit-exact, moments to 1e-12 of the column mass (both sum fp32 per 8 rows and
    fp64 across, in different fp64 orders). Ragged D (not a multiple of 128), ragged n, an offset
    staging column, multi-hot annotation rows; called twice (accumulation, reused workspace)."""
    from proteus_b200 import kernels as KN
    g = torch.Generator(device=DEV).manual_seed(D + n)
    B, levels = 5, [2, 3, 4][:NL] if NL > 1 else [3]
    t = torch.randn(n, D, device=DEV, generator=g) / torch.sqrt((torch.randn(n, D, device=DEV, generator=g) ** 2
                                                                 + torch.randn(n, D, device=DEV, generator=g) ** 2) / 2)
    X = (t * (torch.rand(D, device=DEV, generator=g) + 0.5) + torch.randn(D, device=DEV, generator=g) * 0.5)
    X = X.to(torch.bfloat16)
    qs = torch.tensor([0.5, 0.9, 0.99, 0.999, 0.9999], device=DEV)
    E0 = torch.quantile(X[:4096].float(), qs, dim=0).T.contiguous()
    E1 = torch.quantile(-X[:4096].float(), qs, dim=0).T.contiguous()
    ldx = col0 + ((n + 63) // 64) * 64 + 64
    XT = torch.full((D, ldx), float("nan"), device=DEV, dtype=torch.bfloat16)  # garbage outside the rows
    KN.gather_transpose(X, torch.arange(n, dtype=torch.int32, device=DEV), XT, col0)
    A_pad = max(16, -(-A // 16) * 16)
    n_pad = max(128, -(-n // 128) * 128)
    annT = torch.zeros(A_pad, n_pad, dtype=torch.int8, device=DEV)
    lab = torch.randint(0, A, (n, 3), device=DEV, generator=g)
    keep = torch.rand(n, 3, device=DEV, generator=g) < torch.tensor([1.0, 0.4, 0.2], device=DEV)
    for c in range(3):
        rows = torch.nonzero(keep[:, c]).squeeze(1)
        annT[lab[rows, c], rows] = 1
    assert KN.stats_enrich_supported(torch.bfloat16, B, NL, A_pad)
    want = [torch.zeros(D, dtype=torch.float64, device=DEV), torch.zeros(D, dtype=torch.float64, device=DEV),
            torch.zeros(2, D, B, dtype=torch.int64, device=DEV), torch.zeros(2 * NL * D, A, dtype=torch.int64, device=DEV)]
    got = [torch.zeros_like(x) for x in want]
    masks = torch.zeros(2 * NL * D * n_pad, dtype=torch.int8, device=DEV)
    ws = KN.StatsEnrichWorkspace(DEV)
    M = 2 * NL * D
    M_pad = -(-M // 128) * 128
    mpad = torch.zeros(M_pad * n_pad, dtype=torch.int8, device=DEV)
    for _ in range(2):
        KN.sub_stats_into(XT, col0, n, E0, E1, levels, want[0], want[1], want[2], masks, n_pad)
        mpad[:M * n_pad].copy_(masks)
        out = torch.zeros(M_pad, A, dtype=torch.int64, device=DEV)
        KN.count_gemm_i8(mpad.view(M_pad, n_pad), annT, out, A)
        want[3] += out[:M]
        KN.sub_stats_enrich_into(XT, col0, n, E0, E1, levels, got[0], got[1], got[2], annT, got[3], A, ws)
    torch.cuda.synchronize()
    assert torch.equal(got[2], want[2]), "bin masses differ"
    assert torch.equal(got[3], want[3]), f"contingencies differ in {int((got[3] != want[3]).sum())} entries"
    mass = torch.sqrt(n * want[1]) + 1e-300
    assert bool(((got[0] - want[0]).abs() <= 1e-12 * mass).all())
    assert bool(((got[1] - want[1]).abs() <= 1e-12 * want[1]).all())
    assert int(want[3].sum()) > 0
