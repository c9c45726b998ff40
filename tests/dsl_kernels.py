"""Enigma DSL kernels written the way the reference's callers write them.

Each follows the algorithm of one reference example or test kernel (cited),
expressed against this package's public API.  The tests compile them with
enigma.compile, check what the recognizer bound, and (on a GPU) run them
through MetalRuntime.execute against the CPU oracle.
"""
import enigma
from enigma.tensor import Tensor, tensor_composition, tensor_zipped_divide


# ---------------------------------------------------------------- RMSNorm (TV layout)
# examples/benchmark_rmsnorm.py:31-84: one threadgroup per row, a TV layout of
# `threads` x `values`, simd_sum -> threadgroup scratch -> simd_sum, rsqrt.
def make_rmsnorm(rows, n, threads, values, eps, dtype="float"):
    tiler, tv = enigma.make_layout_tv(enigma.make_ordered_layout((threads,), order=(0,)),
                                      enigma.make_ordered_layout((values,), order=(0,)))

    @enigma.kernel
    def rmsnorm_kernel(gX, gW, gOut, tv_layout, tiler_mn):
        tidx, _, _ = enigma.arch.thread_idx()
        row, _, _ = enigma.arch.block_idx()
        x_row = gX[((None, None), row)][(0, None)]
        y_row = gOut[((None, None), row)][(0, None)]
        w_all = gW[(None,)]
        mine_x = tensor_composition(x_row, tv_layout, tiler_mn)[(tidx, None)]
        mine_y = tensor_composition(y_row, tv_layout, tiler_mn)[(tidx, None)]
        mine_w = tensor_composition(w_all, tv_layout, tiler_mn)[(tidx, None)]
        xv = mine_x.load()
        wv = mine_w.load()
        part = enigma.simd_sum(xv * xv)
        scratch = enigma.threadgroup_alloc("float", 32)
        lane = enigma.thread_index_in_simdgroup()
        warp = enigma.simdgroup_index_in_threadgroup()
        enigma.store_if(scratch, warp, part, enigma.cmp_eq(lane, 0))
        enigma.barrier()
        v = enigma.load_if(scratch, lane, enigma.cmp_ult(lane, enigma.simdgroups_per_threadgroup()),
                           default=0.0)
        total = enigma.simd_sum(v)
        inv = enigma.rsqrt(total / float(n) + eps)
        mine_y.store(xv * inv * wv)

    @enigma.jit
    def rmsnorm_jit(mX, mW, mOut):
        gX = tensor_zipped_divide(mX, (1, tiler[0]))
        gOut = tensor_zipped_divide(mOut, (1, tiler[0]))
        gW = tensor_zipped_divide(mW, tiler)
        t = enigma.size(tv, mode=[0])
        rmsnorm_kernel(gX, gW, gOut, tv, tiler).launch(grid=(rows * t, 1, 1), block=(t, 1, 1))

    mX = Tensor("X", 0, dtype, enigma.Layout((rows, n), (n, 1)))
    mW = Tensor("W", 1, dtype, enigma.Layout((n,), (1,)))
    mOut = Tensor("Out", 2, dtype, enigma.Layout((rows, n), (n, 1)))
    return rmsnorm_jit, (mX, mW, mOut)


# ---------------------------------------------------------------- GQA decode attention
# examples/benchmark_sdpa.py:48-158: threadgroup per (token, kv head), QMUL q heads
# per kv head, simdgroups stride the KV tokens, online softmax, cross-simdgroup merge.
def make_sdpa_gqa(tokens, q_heads, kv_heads, head_dim, kv_tokens, n_sg=4):
    qmul = q_heads // kv_heads
    thr = n_sg * 32
    tiler_d, tv_d = enigma.make_layout_tv(enigma.make_ordered_layout((32,), order=(0,)),
                                          enigma.make_ordered_layout((2,), order=(0,)))

    def head_vec(base, lane):
        t = Tensor("Q", 0, "float", enigma.Layout(head_dim, 1), base_offset=base)
        tiled = tensor_zipped_divide(t, tiler_d)
        return tensor_composition(tiled[(None,)], tv_d, tiler_d)[(lane, None)].load()

    @enigma.kernel
    def sdpa_gqa(mQ, mKV, mM0, mO):
        qt = enigma.threadgroup_position_in_grid("x")
        h = enigma.threadgroup_position_in_grid("y")
        lane = enigma.thread_index_in_simdgroup()
        sg = enigma.simdgroup_index_in_threadgroup()
        q = [head_vec(qt * (q_heads * head_dim) + h * (qmul * head_dim) + g * head_dim, lane)
             for g in enigma.range_constexpr(qmul)]
        m = [mM0[h * qmul + g] for g in enigma.range_constexpr(qmul)]
        l = [enigma.where(enigma.metal_cast(0.0, "float"), enigma.metal_cast(1.0, "float"),
                          enigma.cmp_eq(sg, 0)) for _ in range(qmul)]
        ox = [enigma.metal_cast(0.0, "float") for _ in range(qmul)]
        oy = [enigma.metal_cast(0.0, "float") for _ in range(qmul)]
        for it in enigma.range(kv_tokens // n_sg):
            base = h * kv_tokens * 2 * head_dim + (it * n_sg + sg) * 2 * head_dim
            kv = enigma.make_float2(mKV[base + lane * 2], mKV[base + lane * 2 + 1])
            vx = mKV[base + head_dim + lane * 2]
            vy = mKV[base + head_dim + lane * 2 + 1]
            for g in enigma.range_constexpr(qmul):
                s = enigma.simd_sum(enigma.dot(q[g], kv))
                mn = enigma.fmax(m[g], s)
                a = enigma.exp(m[g] - mn)
                p = enigma.exp(s - mn)
                l[g] = enigma.fma(l[g], a, p)
                m[g] = mn
                ox[g] = enigma.fma(vx, p, ox[g] * a)
                oy[g] = enigma.fma(vy, p, oy[g] * a)
        shared = enigma.threadgroup_alloc("float", 2 * qmul * n_sg)
        for g in enigma.range_constexpr(qmul):
            enigma.store_if(shared, g * n_sg + sg, m[g], enigma.cmp_eq(lane, 0))
        enigma.barrier()
        for g in enigma.range_constexpr(qmul):
            out = ox[g] / l[g]
            mO[qt * q_heads * head_dim + h * qmul * head_dim + g * head_dim + lane * 2] = out
            mO[qt * q_heads * head_dim + h * qmul * head_dim + g * head_dim + lane * 2 + 1] = \
                oy[g] / l[g]

    @enigma.jit
    def sdpa_jit(mQ, mKV, mM0, mO):
        sdpa_gqa(mQ, mKV, mM0, mO).launch(grid=(tokens * thr, kv_heads, 1), block=(thr, 1, 1))

    args = (Tensor("Q", 0, "float", enigma.Layout(tokens * q_heads * head_dim, 1)),
            Tensor("KV", 1, "float", enigma.Layout(kv_heads * kv_tokens * 2 * head_dim, 1)),
            Tensor("M0", 2, "float", enigma.Layout(q_heads, 1)),
            Tensor("O", 3, "float", enigma.Layout(tokens * q_heads * head_dim, 1)))
    return sdpa_jit, args, thr


# ---------------------------------------------------------------- FlashAttention-1 rows
# examples/showcase_attention.py:31-91: one thread per query row, KV tiles of BC keys,
# carried (m, l, o[0..3]) with 1/sqrt(D) scaling; D = 4.
def make_fa(n_keys, bc=16):
    D = 4
    nt = n_keys // bc

    def body(Q, K, V, O, row):
        d = enigma.metal_cast(D, "uint")
        qb = row * d
        qv = enigma.make_float4(Q[qb], Q[qb + 1], Q[qb + 2], Q[qb + 3])
        sc = enigma.rsqrt(enigma.metal_cast(D, "float"))
        neg = enigma.metal_cast(-1e30, "float")
        z = enigma.metal_cast(0, "float")
        with enigma.for_range(0, enigma.metal_cast(nt, "int"), init=[neg, z, z, z, z, z]) as (t, c):
            tb = enigma.metal_cast(t, "uint") * enigma.metal_cast(bc, "uint") * d
            s = []
            for j in range(bc):
                kb = tb + enigma.metal_cast(j * D, "uint")
                s.append(enigma.dot(qv, enigma.make_float4(K[kb], K[kb + 1], K[kb + 2],
                                                           K[kb + 3])) * sc)
            mt = s[0]
            for x in s[1:]:
                mt = enigma.fmax(mt, x)
            mn = enigma.fmax(c[0], mt)
            a = enigma.exp(c[0] - mn)
            ps = [enigma.exp(x - mn) for x in s]
            tot = ps[0]
            for p in ps[1:]:
                tot = tot + p
            o = [a * c[2 + i] for i in range(4)]
            for j in range(bc):
                vb = tb + enigma.metal_cast(j * D, "uint")
                o = [enigma.fma(ps[j], V[vb + i], o[i]) for i in range(4)]
            c[1] = a * c[1] + tot
            c[0] = mn
            for i in range(4):
                c[2 + i] = o[i]
        inv = enigma.metal_cast(1, "float") / c[1]
        for i in range(4):
            O[row * d + i] = c[2 + i] * inv

    @enigma.kernel
    def fa_naive(Q: enigma.f32, K: enigma.f32, V: enigma.f32, O: enigma.f32):
        body(Q, K, V, O, enigma.thread_position_in_grid)

    return fa_naive


# ---------------------------------------------------------------- FlashAttention, any D
# The showcase body (examples/showcase_attention.py:31-91) generalised the way a caller
# writes it for config 4: D/4 float4 chunks per dot, (m, l, o[0..D-1]) carried, one
# query row per thread; threadgroups along y pick the (batch, head) slice of a dense
# [B*H, S, D] buffer.  causal=True masks key > query with where(s, -1e30, key > row).
def _fa_any_body(Q, K, V, O, row, bh, seq_q, seq_k, D, bc, causal, out_dtype):
    def u(v):
        return enigma.metal_cast(v, "uint")

    def f(x):
        return enigma.metal_cast(x, "float")

    qb = bh * u(seq_q * D) + row * u(D)
    kvb = bh * u(seq_k * D)
    qv = [enigma.make_float4(*[f(Q[qb + u(4 * c + i)]) for i in range(4)])
          for c in range(D // 4)]
    sc = enigma.rsqrt(enigma.metal_cast(D, "float"))
    neg = enigma.metal_cast(-1e30, "float")
    z = enigma.metal_cast(0, "float")
    with enigma.for_range(0, enigma.metal_cast(seq_k // bc, "int"),
                          init=[neg, z] + [z] * D) as (t, c):
        tb = kvb + enigma.metal_cast(t, "uint") * u(bc * D)
        s = []
        for j in range(bc):
            kb = tb + u(j * D)
            acc = None
            for cc in range(D // 4):
                kv = enigma.make_float4(*[f(K[kb + u(4 * cc + i)]) for i in range(4)])
                d = enigma.dot(qv[cc], kv)
                acc = d if acc is None else acc + d
            x = acc * sc
            if causal:
                key = enigma.metal_cast(t, "uint") * u(bc) + u(j)
                x = enigma.where(x, neg, enigma.cmp_ugt(key, row))
            s.append(x)
        mt = s[0]
        for x in s[1:]:
            mt = enigma.fmax(mt, x)
        mn = enigma.fmax(c[0], mt)
        a = enigma.exp(c[0] - mn)
        ps = [enigma.exp(x - mn) for x in s]
        tot = ps[0]
        for p in ps[1:]:
            tot = tot + p
        o = [a * c[2 + i] for i in range(D)]
        for j in range(bc):
            vb = tb + u(j * D)
            o = [enigma.fma(ps[j], f(V[vb + u(i)]), o[i]) for i in range(D)]
        c[1] = a * c[1] + tot
        c[0] = mn
        for i in range(D):
            c[2 + i] = o[i]
    inv = enigma.metal_cast(1, "float") / c[1]
    for i in range(D):
        O[qb + u(i)] = enigma.metal_cast(c[2 + i] * inv, out_dtype)


def make_fa_heads(seq, D, causal, bc=16, dtype="bfloat"):
    """@enigma.kernel form: dispatch with grid=(seq, B*H, 1), threads=(BR, 1, 1)."""
    ann = enigma.bf16 if dtype == "bfloat" else enigma.f32

    def body(Q, K, V, O):
        row = enigma.thread_position_in_grid_xyz("x")
        bh = enigma.threadgroup_position_in_grid("y")
        _fa_any_body(Q, K, V, O, row, bh, seq, seq, D, bc, causal, dtype)

    if causal:
        @enigma.kernel
        def fa_causal(Q: ann, K: ann, V: ann, O: ann):
            body(Q, K, V, O)
        return fa_causal

    @enigma.kernel
    def fa_heads(Q: ann, K: ann, V: ann, O: ann):
        body(Q, K, V, O)
    return fa_heads


# ---------------------------------------------------------------- FlashAttention, TV launcher
# examples/showcase_attention.py:94-131: the same body launched from a TV layout,
# thread layout (BR, 1) x value layout (1, D), grid from zipped_divide of Q by the tiler.
# With heads > 1 the launcher adds a y extent of B*H over per-head (S, D) tensors.
def make_fa_tv(M, N, D, BR=32, bc=16, heads=1, causal=False, dtype="float"):
    from enigma._tracing import Tensor as TTensor

    @enigma.kernel
    def fa_tv_kernel(Q, K, V, O):
        Qt = TTensor(Q.name, Q.buffer_index, Q.metal_dtype)
        Kt = TTensor(K.name, K.buffer_index, K.metal_dtype)
        Vt = TTensor(V.name, V.buffer_index, V.metal_dtype)
        Ot = TTensor(O.name, O.buffer_index, O.metal_dtype)
        tidx, _, _ = enigma.arch.thread_idx()
        bidx, _, _ = enigma.arch.block_idx()
        bdim, _, _ = enigma.arch.block_dim()
        row = bidx * bdim + tidx
        bh = enigma.threadgroup_position_in_grid("y") if heads > 1 else 0
        _fa_any_body(Qt, Kt, Vt, Ot, row, bh, M, N, D, bc, causal, dtype)

    @enigma.jit
    def fa_tv(mQ, mK, mV, mO):
        thr_layout = enigma.make_ordered_layout((BR, 1), order=(1, 0))
        val_layout = enigma.make_ordered_layout((1, D), order=(1, 0))
        tiler_mn, tv_layout = enigma.make_layout_tv(thr_layout, val_layout)
        gQ = tensor_zipped_divide(mQ, tiler_mn)
        num_blocks = enigma.size(gQ, mode=[1])
        threads = enigma.size(tv_layout, mode=[0])
        fa_tv_kernel(mQ, mK, mV, mO).launch(grid=(num_blocks * threads, heads, 1),
                                            block=(threads, 1, 1))

    args = (Tensor("Q", 0, dtype, enigma.Layout((M, D), (D, 1))),
            Tensor("K", 1, dtype, enigma.Layout((N, D), (D, 1))),
            Tensor("V", 2, dtype, enigma.Layout((N, D), (D, 1))),
            Tensor("O", 3, dtype, enigma.Layout((M, D), (D, 1))))
    return fa_tv, args


# ---------------------------------------------------------------- K = 4 matmul / gemm
# tests/metal/test_gemm_matmul_runtime.py:20-60
def make_k4(n_cols, accumulate):
    def body(A, B, C):
        row = enigma.thread_position_in_grid_xyz("y")
        col = enigma.thread_position_in_grid_xyz("x")
        n = enigma.metal_cast(n_cols, "uint")
        k = enigma.metal_cast(4, "uint")
        av = enigma.make_float4(*[A[row * k + i] for i in range(4)])
        bv = enigma.make_float4(*[B[col + n * i] for i in range(4)])
        idx = row * n + col
        C[idx] = enigma.dot(av, bv) + C[idx] if accumulate else enigma.dot(av, bv)

    if accumulate:
        @enigma.kernel
        def gemm_k4(A: enigma.f32, B: enigma.f32, C: enigma.f32):
            body(A, B, C)
        return gemm_k4

    @enigma.kernel
    def matmul_k4(A: enigma.f32, B: enigma.f32, C: enigma.f32):
        body(A, B, C)
    return matmul_k4


# ---------------------------------------------------------------- enigma.gemm tile op
# tests/metal/test_new_features_runtime.py:25-56: stage A and B into threadgroup tiles,
# one enigma.gemm into a zero-filled register tile, store the tile.
def make_tile_gemm(M, N, K, transpose_A=False, transpose_B=False):
    @enigma.kernel
    def tile_gemm(A: enigma.f32, B: enigma.f32, Out: enigma.f32):
        A_s = enigma.threadgroup_alloc("float", M * K)
        B_s = enigma.threadgroup_alloc("float", K * N)
        for i in range(M * K):
            A_s[i] = A[i]
        for i in range(K * N):
            B_s[i] = B[i]
        enigma.barrier("mem_threadgroup")
        C = enigma.register_tensor((M, N), dtype="float", fill=0.0)
        enigma.gemm(A_s, B_s, C, M=M, N=N, K=K, transpose_A=transpose_A,
                    transpose_B=transpose_B)
        for m in range(M):
            for n in range(N):
                Out[m * N + n] = C[m, n]

    return tile_gemm


# ---------------------------------------------------------------- async-copy tiled GEMM
# examples/async_copy_gemm.py:32-79: A/B tiles staged into threadgroup memory with 2-D
# async copies, K loop over tiles.
def make_async_gemm(m, n, k, tm=32, tn=32, tk=16, dtype="float"):
    ann = enigma.bf16 if dtype == "bfloat" else enigma.f32

    @enigma.kernel
    def gemm_async(A: ann, B: ann, C: ann):
        tg = enigma.threadgroup_position_in_grid()
        cols = enigma.metal_cast(n // tn, "uint")
        bx, by = tg / cols, tg % cols
        sg = enigma.simdgroup_index_in_threadgroup()
        a_tile = enigma.threadgroup_alloc(dtype, tm * tk)
        b_tile = enigma.threadgroup_alloc(dtype, tk * tn)
        acc = enigma.register_tensor((2, 2), dtype="float", fill=0.0)
        zero = enigma.metal_cast(0, "uint")
        kc = enigma.metal_cast(k, "uint")
        nc = enigma.metal_cast(n, "uint")
        for kt in range(k // tk):
            koff = enigma.metal_cast(kt, "uint") * enigma.metal_cast(tk, "uint")
            with enigma.if_(enigma.cmp_eq(sg, 0)) as (then_b, _):
                with then_b:
                    ea = enigma.async_copy_2d_d2t(a_tile, zero, tk, A, bx * tm * kc + koff, kc,
                                                  tk, tm)
                    eb = enigma.async_copy_2d_d2t(b_tile, zero, tn, B, koff * nc + by * tn, nc,
                                                  tn, tk)
                    enigma.async_copy_wait(ea, eb)
            enigma.barrier()
        C[(bx * tm) * nc + by * tn + enigma.thread_position_in_threadgroup()] = acc[0, 0]

    return gemm_async


# ---------------------------------------------------------------- Qwen single-layer decode
# examples/qwen_megakernel.py:41-269: one threadgroup, phases separated by device barriers.
def make_qwen(H, INTER, QH, KVH, CACHE_TOTAL, eps=1e-6, TG=256):
    HD = H // QH
    G = QH // KVH
    scale = 1.0 / float(HD) ** 0.5

    def u(v):
        return enigma.metal_cast(v, "uint")

    def rmsnorm(X, W, Y, dim, tid):
        lane = enigma.thread_index_in_simdgroup()
        sg = enigma.simdgroup_index_in_threadgroup()
        z = enigma.metal_cast(0, "float")
        with enigma.for_range(0, dim // TG, init=[z]) as (j, c):
            v = X[tid + u(j) * u(TG)]
            c[0] = c[0] + v * v
        part = enigma.simd_sum(c[0])
        scratch = enigma.threadgroup_alloc("float", 32)
        enigma.store_if(scratch, sg, part, enigma.cmp_eq(lane, 0))
        enigma.barrier()
        tot = enigma.simd_sum(enigma.load_if(scratch, lane,
                                             enigma.cmp_ult(lane, enigma.simdgroups_per_threadgroup()),
                                             default=0.0))
        r = enigma.rsqrt(tot / float(dim) + eps)
        with enigma.for_range(0, dim // TG) as j:
            idx = tid + u(j) * u(TG)
            Y[idx] = (X[idx] * r) * W[idx]

    def matvec(X, W, Out, rows, cols, tid, res=None, Wu=None):
        with enigma.for_range(0, (rows + TG - 1) // TG) as ch:
            row = tid + u(ch) * u(TG)
            with enigma.if_(enigma.cmp_ult(row, u(rows))):
                z = enigma.metal_cast(0, "float")
                init = [z, z] if Wu is not None else [z]
                with enigma.for_range(0, cols, init=init) as (i, c):
                    xv = X[u(i)]
                    c[0] = enigma.fma(W[row * u(cols) + u(i)], xv, c[0])
                    if Wu is not None:
                        c[1] = enigma.fma(Wu[row * u(cols) + u(i)], xv, c[1])
                if Wu is not None:
                    one = enigma.metal_cast(1, "float")
                    Out[row] = (c[0] * (one / (one + enigma.exp(-c[0])))) * c[1]
                else:
                    Out[row] = c[0] + res[row] if res is not None else c[0]

    def head_norm_rope(src, w, cs, sn, dst, nh, tid):
        with enigma.if_(enigma.cmp_ult(tid, u(nh))):
            base = tid * u(HD)
            z = enigma.metal_cast(0, "float")
            with enigma.for_range(0, HD, init=[z]) as (k, c):
                v = src[base + u(k)]
                c[0] = c[0] + v * v
            sc = enigma.rsqrt(c[0] / float(HD) + eps)
            with enigma.for_range(0, HD) as k:
                dst[base + u(k)] = src[base + u(k)] * sc * w[u(k)]
            with enigma.for_range(0, HD // 2) as k:
                lo_i, hi_i = base + u(k), base + u(k) + u(HD // 2)
                lo, hi = dst[lo_i], dst[hi_i]
                dst[lo_i] = lo * cs[u(k)] - hi * sn[u(k)]
                dst[hi_i] = hi * cs[u(k) + u(HD // 2)] + lo * sn[u(k) + u(HD // 2)]

    def sdpa(Q, K, V, O, tid):
        with enigma.if_(enigma.cmp_ult(tid, u(QH))):
            kvh = tid / u(G)
            neg, z = enigma.metal_cast(-1e30, "float"), enigma.metal_cast(0, "float")
            with enigma.for_range(0, CACHE_TOTAL, init=[neg, z]) as (pos, c):
                with enigma.for_range(0, HD, init=[z]) as (d, dc):
                    dc[0] = enigma.fma(Q[tid * u(HD) + u(d)],
                                       K[kvh * u(CACHE_TOTAL * HD) + u(pos) * u(HD) + u(d)], dc[0])
                s = dc[0] * scale
                mn = enigma.fmax(c[0], s)
                c[1] = c[1] * enigma.exp(c[0] - mn) + enigma.exp(s - mn)
                c[0] = mn
            m_fin = c[0]
            inv_l = enigma.metal_cast(1, "float") / c[1]
            with enigma.for_range(0, HD) as d:
                with enigma.for_range(0, CACHE_TOTAL, init=[z]) as (pos, vc):
                    with enigma.for_range(0, HD, init=[z]) as (d2, dc2):
                        dc2[0] = enigma.fma(Q[tid * u(HD) + u(d2)],
                                            K[kvh * u(CACHE_TOTAL * HD) + u(pos) * u(HD) + u(d2)],
                                            dc2[0])
                    p = enigma.exp(dc2[0] * scale - m_fin) * inv_l
                    vc[0] = vc[0] + p * V[kvh * u(CACHE_TOTAL * HD) + u(pos) * u(HD) + u(d)]
                O[tid * u(HD) + u(d)] = vc[0]

    @enigma.kernel
    def qwen_fused(X: enigma.f32, w_norm: enigma.f32, Wq: enigma.f32, Wk: enigma.f32,
                   Wv: enigma.f32, w_q_norm: enigma.f32, w_k_norm: enigma.f32,
                   cos_pos: enigma.f32, sin_pos: enigma.f32, K_cache: enigma.f32,
                   V_cache: enigma.f32, Wo: enigma.f32, w_post: enigma.f32, Wg: enigma.f32,
                   Wu: enigma.f32, Wd: enigma.f32, norm_buf: enigma.f32, q_buf: enigma.f32,
                   k_buf: enigma.f32, v_buf: enigma.f32, attn_buf: enigma.f32,
                   mlp_buf: enigma.f32, post_buf: enigma.f32, q_rope_buf: enigma.f32,
                   k_rope_buf: enigma.f32, Out: enigma.f32):
        tid = enigma.thread_position_in_threadgroup()
        rmsnorm(X, w_norm, norm_buf, H, tid)
        enigma.barrier("mem_device_and_threadgroup")
        matvec(norm_buf, Wq, q_buf, QH * HD, H, tid)
        matvec(norm_buf, Wk, k_buf, KVH * HD, H, tid)
        matvec(norm_buf, Wv, v_buf, KVH * HD, H, tid)
        enigma.barrier("mem_device_and_threadgroup")
        head_norm_rope(q_buf, w_q_norm, cos_pos, sin_pos, q_rope_buf, QH, tid)
        head_norm_rope(k_buf, w_k_norm, cos_pos, sin_pos, k_rope_buf, KVH, tid)
        enigma.barrier("mem_device_and_threadgroup")
        sdpa(q_rope_buf, K_cache, V_cache, attn_buf, tid)
        enigma.barrier("mem_device_and_threadgroup")
        matvec(attn_buf, Wo, norm_buf, H, QH * HD, tid, res=X)
        enigma.barrier("mem_device_and_threadgroup")
        rmsnorm(norm_buf, w_post, post_buf, H, tid)
        enigma.barrier("mem_device_and_threadgroup")
        matvec(post_buf, Wg, mlp_buf, INTER, H, tid, Wu=Wu)
        enigma.barrier("mem_device_and_threadgroup")
        matvec(mlp_buf, Wd, Out, H, INTER, tid, res=norm_buf)

    return qwen_fused


# ---------------------------------------------------------------- TV elementwise add
# examples/vector_add_tv.py:13-55: (4,64) threads x (4,4) values per 64x... tile.
def make_tv_add(M, N, dtype="float"):
    @enigma.kernel
    def add_kernel(gA, gB, gC, tv_layout, tiler):
        tidx, _, _ = enigma.arch.thread_idx()
        bidx, _, _ = enigma.arch.block_idx()
        frag = [tensor_composition(g[((None, None), bidx)], tv_layout, tiler)[(tidx, None)]
                for g in (gA, gB, gC)]
        frag[2].store(frag[0].load() + frag[1].load())

    @enigma.jit
    def elementwise_add(mA, mB, mC):
        tiler, tv = enigma.make_layout_tv(enigma.make_ordered_layout((4, 64), order=(1, 0)),
                                          enigma.make_ordered_layout((4, 4), order=(1, 0)))
        gs = [tensor_zipped_divide(m, tiler) for m in (mA, mB, mC)]
        blocks, threads = enigma.size(gs[0], mode=[1]), enigma.size(tv, mode=[0])
        add_kernel(*gs, tv, tiler).launch(grid=(blocks * threads, 1, 1), block=(threads, 1, 1))

    args = tuple(Tensor(n, i, dtype, enigma.Layout((M, N), (N, 1))) for i, n in enumerate("ABC"))
    return elementwise_add, args


def make_naive_binary(op):
    @enigma.kernel
    def binary(A: enigma.f32, B: enigma.f32, C: enigma.f32):
        i = enigma.thread_position_in_grid
        C[i] = op(A[i], B[i])
    return binary


# ---------------------------------------------------------------- RMSNorm with runtime eps
# One threadgroup per row, strided loop over the row (the layout of the Qwen layer's
# _rmsnorm, qwen_megakernel.py:41-66), eps given as a Scalar parameter or a function constant.
def make_rmsnorm_runtime_eps(hidden, mode, TG=256):
    def u(v):
        return enigma.metal_cast(v, "uint")

    def body(X, W, Y, eps):
        row = enigma.threadgroup_position_in_grid("x")
        tid = enigma.thread_position_in_threadgroup()
        base = row * u(hidden)
        lane = enigma.thread_index_in_simdgroup()
        sg = enigma.simdgroup_index_in_threadgroup()
        z = enigma.metal_cast(0, "float")
        with enigma.for_range(0, hidden // TG, init=[z]) as (j, c):
            v = X[base + tid + u(j) * u(TG)]
            c[0] = c[0] + v * v
        scratch = enigma.threadgroup_alloc("float", 32)
        enigma.store_if(scratch, sg, enigma.simd_sum(c[0]), enigma.cmp_eq(lane, 0))
        enigma.barrier()
        tot = enigma.simd_sum(enigma.load_if(scratch, lane, enigma.cmp_ult(
            lane, enigma.simdgroups_per_threadgroup()), default=0.0))
        r = enigma.rsqrt(tot / float(hidden) + eps)
        with enigma.for_range(0, hidden // TG) as j:
            i = tid + u(j) * u(TG)
            Y[base + i] = X[base + i] * r * W[i]

    if mode == "scalar":
        @enigma.kernel
        def rmsnorm_scalar_eps(X: enigma.f32, W: enigma.f32, eps: enigma.Scalar(enigma.f32),
                               Y: enigma.f32):
            body(X, W, Y, eps)
        return rmsnorm_scalar_eps

    @enigma.kernel
    def rmsnorm_const_eps(X: enigma.f32, W: enigma.f32, Y: enigma.f32):
        body(X, W, Y, enigma.function_constant("float", 0))
    return rmsnorm_const_eps
