"""Replays the library's job entry points on the oracle's CPU job models over
CPU tensors — TEST INFRASTRUCTURE: ``install`` swaps ``cormorant_b200.ops``'
kernel calls for the models, so ``GpuSimulator``'s host logic (registers,
strides, buffers, states, fusion) runs without a GPU.  Used by the
``cpu_ops`` fixture and by the multi-process (gloo) tests, whose ranks are
spawned processes without pytest fixtures."""
import numpy as np


def install(setattr_fn):
    """Patch ops.* (and GpuSimulator's workspace query) through
    ``setattr_fn(obj, name, value)``; returns the GpuSimulator class."""
    import torch

    from cormorant_b200 import ops
    from cormorant_b200._lib import F_ACT_RELU, F_ACT_RELU6, F_WRAP32
    from cormorant_b200.simulator import GpuSimulator
    from oracle import spec

    def np16(t):
        return t.numpy() if t is not None else None

    def rowops(a, b, c, p, *, op, n, rows=1, blocks=1, a_s1=0, a_s2=0, b_s1=0, b_s2=0, c_s1=0, c_s2=0, eps=0, aux=0,
               bq_sh=0, win_lo=0, win_hi=0xFFFFFFFF, a_off=0, b_off=0, c_off=0, p_off=0):
        regions, base, addr = {}, 0, {}
        for nm, t, off in (("a", a, a_off), ("b", b, b_off), ("c", c, c_off), ("p", p, p_off)):
            if t is None:
                addr[nm] = 0
                continue
            st = t.untyped_storage()
            key = st.data_ptr()
            if key not in regions:
                regions[key] = (base, st)
                base += (st.nbytes() + 255) // 256 * 256 + 256
            addr[nm] = regions[key][0] + (t.data_ptr() - key) + off
        mem = np.zeros(base, np.uint8)
        for b0, st in regions.values():
            mem[b0:b0 + st.nbytes()] = np.frombuffer(bytes(st), np.uint8)
        m = spec.RowOpsMem(mem)
        spec.rowops_job(m, op, n, rows, blocks, addr["a"], a_s1, a_s2, addr["b"], b_s1, b_s2, addr["c"], c_s1, c_s2,
                        addr["p"], eps, aux, bq_sh, win_lo, win_hi)
        cst = c.untyped_storage()
        b0 = regions[cst.data_ptr()][0]
        cst.copy_(torch.frombuffer(bytearray(m.buf[b0:b0 + cst.nbytes()].tobytes()), dtype=torch.uint8).untyped_storage())

    def matmul(a, b, c, *, n, k, m, batch=1, a_batch_stride=0, b_batch_stride=0, c_batch_stride=0, b_packed=0,
               gemv_kw=0, flags=0, workspace=None, post=None):
        assert post is None
        spec.matmul_job(np16(a), np16(b), np16(c), n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride,
                        b_packed, gemv_kw, wrap=bool(flags & F_WRAP32))

    def mulact_pairs(y, sa, sc):
        """Gate / up pairs of 16-column blocks -> the row-ops MULACT of each pair."""
        n, m = y.shape
        g = y.reshape(n, m // 32, 2, 16)[:, :, 0, :].reshape(n, m // 2)
        u = y.reshape(n, m // 32, 2, 16)[:, :, 1, :].reshape(n, m // 2)
        out = np.empty((n, m // 2), np.int64)
        for idx in np.ndindex(out.shape):
            v = spec._rne(spec.silu_q(int(g[idx]) << sa) * int(u[idx]), sc)
            out[idx] = min(max(v, -32768), 32767)
        return out

    def matmul_groups(a, b, outs, widths, *, n, k, batch=1, a_batch_stride=0, b_batch_stride=0, flags=0,
                      workspace=None, mulact=None):
        assert batch == 1
        m = sum(widths) * (2 if mulact is not None else 1)
        y = spec.matmul_raw(np16(a)[:n * k].astype(np.int64).reshape(n, k), np16(b)[:k * m].astype(np.int64).reshape(k, m),
                            wrap=bool(flags & F_WRAP32))
        if mulact is not None:
            np16(outs[0])[:n * m // 2] = mulact_pairs(y, *mulact).reshape(-1)
            return
        c0 = 0
        for o, w in zip(outs, widths):
            np16(o)[:n * w] = y[:, c0:c0 + w].reshape(-1)
            c0 += w

    def split_b_planes(b, *, k, m):
        return (b, None)  # the fake keeps the int16 weight itself

    def matmul_bplanes(a, planes, c, *, n, k, m, batch=1, a_batch_stride=0, c_batch_stride=0, flags=0,
                       workspace=None, outs=None, widths=None, mulact=None):
        assert batch == 1
        y = spec.matmul_raw(np16(a)[:n * k].astype(np.int64).reshape(n, k),
                            np16(planes[0])[:k * m].astype(np.int64).reshape(k, m), wrap=bool(flags & F_WRAP32))
        if mulact is not None:
            np16(outs[0])[:n * m // 2] = mulact_pairs(y, *mulact).reshape(-1)
            return
        if flags & (F_ACT_RELU | F_ACT_RELU6):  # a fused ReLU / Clip(0,6)
            y = np.maximum(y, 0)
            if flags & F_ACT_RELU6:
                y = np.minimum(y, 1536)
        if outs is None:
            np16(c)[:n * m] = y.reshape(-1)
            return
        c0 = 0
        for o, w in zip(outs, widths):
            np16(o)[:n * w] = y[:, c0:c0 + w].reshape(-1)
            c0 += w

    def vectorop(a, b, c, *, size, op, outer=1, a_inc=0, b_inc=0, act=0, alpha=0, smx_cm=0, smx_cfg=0, smx_mask=0):
        spec.vectorop_job(np16(a), np16(b), np16(c), size, op, outer, a_inc, b_inc, act, alpha, smx_cm, smx_cfg,
                          smx_mask)

    def view(t, off, dims, strides):
        a = t.numpy()
        return np.lib.stride_tricks.as_strided(a[off:], shape=tuple(dims), strides=tuple(2 * x for x in strides),
                                               writeable=True)

    def gemm_strided(a, b, c, *, n, k, m, batch=1, lda=None, ldb=None, ldc=None, b_trans=False, a_batch_stride=0,
                     b_batch_stride=0, c_batch_stride=0, flags=0, workspace=None):
        lda, ldc = k if lda is None else lda, m if ldc is None else ldc
        ldb = (k if b_trans else m) if ldb is None else ldb
        A = view(a, 0, (batch, n, k), (a_batch_stride, lda, 1))
        Bm = view(b, 0, (batch, m, k) if b_trans else (batch, k, m), (b_batch_stride, ldb, 1))
        if b_trans:
            Bm = Bm.transpose(0, 2, 1)
        out = view(c, 0, (batch, n, m), (c_batch_stride, ldc, 1))
        out[...] = spec.matmul_raw(A.astype(np.int64), Bm.astype(np.int64), bool(flags & F_WRAP32))
        return workspace

    def copy_nd(src, dst, dims, src_strides, dst_strides, *, src_off=0, dst_off=0):
        v = view(src, src_off, dims, src_strides).copy()
        out = view(dst, dst_off, dims, dst_strides)
        out[...] = v

    def llm_attn_softmax(s, p, tab, ip, *, pos, n, T, G, rows, Q=16, window=0, batch=1, s_stride=None,
                         p_stride=None):
        C = rows
        from oracle import attn as A
        S = s.numpy()[:C * batch * G * T].reshape(C, batch * G * T)
        out = p.numpy()
        tabs = tab.numpy().reshape(G, 65536)
        ipv = ip.numpy()
        nn, _keys = A.attn_keys(pos, n, T, C, Q)
        for col in range(batch * G * T):
            hh, t = (col % (G * T)) // T, col % T
            row = np.zeros(C, np.int64)
            if t < nn:
                nk = pos + t + 1
                j0 = nk - window if (window and nk > window) else 0
                r = S[j0:nk, col].astype(np.int64)
                e = tabs[hh][r.max() - r]
                ssum = 0.0
                for v in e:
                    ssum += v
                row[j0:nk] = np.minimum(np.rint((e / ssum) * ipv[hh]), 32767)
            out[col * C:(col + 1) * C] = row

    def greedy_embed(logits, table, out, ids=None, *, batch, vocab, dim, ld=None):
        lg = logits.numpy()[:batch * (ld or vocab)].reshape(batch, ld or vocab)[:, :vocab]
        nxt = lg.argmax(axis=1)
        out.numpy()[:batch * dim] = table.numpy()[nxt].reshape(-1)
        if ids is not None:
            ids.numpy()[:batch] = nxt

    def llm_decode_attn(qx, kc, vc, tab, ip, o, *, pos, B, KV, G, HD, rows, Q=16, window=0, o_stride=None,
                        prep=None):
        from oracle import attn as A
        C = rows
        if prep is not None:  # the fused AttnPrep: RoPE / re-round by the entries, the cache rows of pos
            ents = lambda t, bc, cnt: np.frombuffer(t.numpy().tobytes()[:16 * (1 if bc else cnt)],  # noqa: E731
                                                    np.uint8).reshape(-1, 16)
            tabw = np.frombuffer(prep["rope"].numpy().tobytes()[:C * 8 * HD], "<i4").astype(np.int64).reshape(C, 2 * HD)
            cs, sn = tabw[pos, :HD], tabw[pos, HD:]
            half = HD // 2

            def rope_rows(x, e, nh):
                x = x.astype(np.int64).reshape(-1, nh, HD)
                rot = np.concatenate([-x[..., half:], x[..., :half]], -1)
                sa = np.broadcast_to(e[:, 8].astype(np.int64) & 63, (nh * HD,)).reshape(nh, HD)
                sb = np.broadcast_to(e[:, 9].astype(np.int64) & 63, (nh * HD,)).reshape(nh, HD)
                sc = np.broadcast_to(e[:, 10].astype(np.int64) & 63, (nh * HD,)).reshape(nh, HD)
                return spec.sat16(spec.rne_shr(((x * cs) << sa) + ((rot * sn) << sb), sc))
            H = KV * G
            q0 = prep["q0"].numpy()[:B * H * HD].reshape(B, H * HD)
            k0 = prep["k0"].numpy()[:B * KV * HD].reshape(B, KV * HD)
            v0 = prep["v0"].numpy()[:B * KV * HD].reshape(B, KV * HD).astype(np.int64)
            qr = rope_rows(q0, ents(prep["pq"], prep["pq_bc"], H * HD), H)          # [B][H][HD]
            kr = rope_rows(k0, ents(prep["pk"], prep["pk_bc"], KV * HD), KV)        # [B][KV][HD]
            if prep["v_direct"]:
                vr = v0
            else:
                e = ents(prep["pv"], prep["pv_bc"], KV * HD)
                sa = np.broadcast_to(e[:, 8].astype(np.int64) & 63, (KV * HD,))
                sc = np.broadcast_to(e[:, 10].astype(np.int64) & 63, (KV * HD,))
                bq = np.broadcast_to(e[:, 4:8].copy().view("<i4").reshape(-1).astype(np.int64), (KV * HD,))
                bq = ((bq << 42) >> 42)
                vr = spec.sat16(spec.rne_shr((v0 << sa) + bq, sc))
            kcn, vcn = kc.numpy(), vc.numpy()
            if pos < C:
                for b in range(B):
                    for g in range(KV):
                        base = ((g * B + b) * C + pos) * HD
                        kcn[base:base + HD] = kr[b, g]
                        vcn[base:base + HD] = vr.reshape(B, KV, HD)[b, g]
            q = np.zeros((KV, B, HD, G), np.int64)
            if pos < C:
                q = qr.reshape(B, KV, G, HD).transpose(1, 0, 3, 2)
        else:
            q = qx.numpy()[:KV * B * HD * G].astype(np.int64).reshape(KV, B, HD, G)
        K = kc.numpy()[:KV * B * C * HD].astype(np.int64).reshape(KV, B, C, HD)
        V = vc.numpy()[:KV * B * C * HD].astype(np.int64).reshape(KV, B, C, HD)
        tabs = tab.numpy().reshape(KV * G, 65536)
        out = o.numpy()
        ost = KV * G * HD if o_stride is None else o_stride
        n, keys = A.attn_keys(pos, 1, 1, C, Q)
        for b in range(B):
            for g in range(KV):
                s = A.kernel_out(K[g, b, :keys] @ q[g, b])                 # [keys][G]
                P = np.zeros((G, C), np.int64)
                if n:
                    nk = pos + 1
                    j0 = nk - window if (window and nk > window) else 0
                    for h in range(G):
                        r = s[j0:nk, h]
                        e = tabs[g * G + h][r.max() - r]
                        ssum = 0.0
                        for v in e:
                            ssum += v
                        P[h, j0:nk] = np.minimum(np.rint((e / ssum) * ip.numpy()[g * G + h]), 32767)
                ob = A.kernel_out(P[:, :keys] @ V[g, b, :keys])            # [G][HD]
                out[b * ost + g * G * HD: b * ost + (g + 1) * G * HD] = ob.reshape(-1)

    setattr_fn(ops, "llm_decode_attn", llm_decode_attn)
    setattr_fn(ops, "llm_attn_softmax", llm_attn_softmax)
    setattr_fn(ops, "greedy_embed", greedy_embed)
    setattr_fn(ops, "gemm_strided", gemm_strided)
    setattr_fn(ops, "copy_nd", copy_nd)
    setattr_fn(ops, "rowops", rowops)

    def rowops_chain(jobs):  # the jobs in order (the library may fuse adjacent ones; the result is the same)
        for j in jobs:
            rowops(j.get("a"), j.get("b"), j.get("c"), j.get("p"),
                   **{k: v for k, v in j.items() if k not in ("a", "b", "c", "p")})
    setattr_fn(ops, "rowops_chain", rowops_chain)
    setattr_fn(ops, "matmul", matmul)
    setattr_fn(ops, "matmul_groups", matmul_groups)
    setattr_fn(ops, "split_b_planes", split_b_planes)
    setattr_fn(ops, "matmul_bplanes", matmul_bplanes)
    setattr_fn(ops, "vectorop", vectorop)
    setattr_fn(GpuSimulator, "_mm_ws", staticmethod(lambda *a: 0))
    return GpuSimulator
