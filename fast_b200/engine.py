"""Autograd-free training step of the TGAT GeneralModel on the fast_b200 kernels.

The reference trains GeneralModel (modules.py:8-70) with PyTorch autograd:
per layer the attention core, then w_out / ReLU / dropout / LayerNorm
(layers.py:213-223), the EdgePredictor (layers.py:31-50) and
BCEWithLogitsLoss (train.py:205-206).  `FusedStep` runs that same forward
and its hand-derived backward as an explicit sequence of kernel launches:

  per layer, forward     gather + time encode -> K|V GEMM -> Q GEMM ->
                         attention -> w_out GEMM(s) -> tail (dropout, ReLU, LayerNorm)
  predictor + loss       src_fc / dst_fc GEMMs -> fused scores + loss + dS, dP
  per layer, backward    tail backward -> w_out grads (bias in the same pass) ->
                         d agg -> attention backward -> K|V grads -> time-encode
                         grads -> Q grads -> input gradient of the layer below

Parameters and their gradients are views of two flat buffers
(`flat_params`, `flat`): gradients go straight into `.grad`, so there is no
autograd graph, no gradient accumulation pass and one memset per step; the
gradient buffer is what data-parallel training all-reduces and `FlatAdam`
updates all parameters in one launch.  w_k / w_v are adjacent rows of one
[2D, K] group (and their biases of one [2D] group), so K and V come from one
GEMM; state_dict names and shapes are unchanged.

Every launch honours device-side row counts (StaticBlock), so the step can
be captured in a CUDA graph.

With node memory (memory.MemoryModel, TGN) the step starts with the memory
updater on the first layer's source rows (memorys.py:270-304): gather of
memory / mailbox / memory time encoding -> the GRU's two products as one
grouped GEMM -> gate kernel; the updated memory is layer 0's node input, and
the backward runs layer 0's input gradient through the gates into the GRU's
weights and the memory time encoder.  `last_memory` keeps the updated memory
for the mailbox writes after the optimizer step (memorys.py:84-142).
"""
import os

import torch

from . import ops

_ALIGN = 64            # flat-buffer segments start on 256-byte boundaries
# FB_FUSED_GATHER=1 gathers layer 0's bf16 projection rows inside the GEMM
# (cp.async row copies from the feature tables by the producer warp) instead
# of materialising them.  Off by default: inside the GEMM's pipeline the row
# copies deliver ~4 bytes per clock per SM, so the gathered K|V projection
# takes ~1.5 ms at config 5's hop 2 against 0.61 ms for the GEMM plus 0.63 ms
# for the gather that writes the rows.
FUSED_GATHER_OFF = os.environ.get("FB_FUSED_GATHER", "0") != "1"


# FB_SIDE_STREAMS=0 keeps every launch of the step on one stream
SIDE_STREAMS = os.environ.get("FB_SIDE_STREAMS", "1") != "0"
# FB_NODE_PRODUCT=0 computes layer 0's node-feature product per edge row
NODE_PRODUCT = os.environ.get("FB_NODE_PRODUCT", "1") != "0"


def pad64(n):
    return (n + 63) // 64 * 64 if n > 0 else 0


class _LayerParams:
    def __init__(self, layer):
        self.L = layer
        self.D = layer.dim_out
        self.dn, self.de, self.dtime = layer.dim_node_feat, layer.dim_edge_feat, layer.dim_time
        self.W_kv = self.b_kv = None
        self.gW_kv = self.gb_kv = None


class FusedStep:
    """Forward + backward + loss of a memoryless transformer_attention
    GeneralModel.  Call `step(blocks, node_table, edge_table, loss_out)`; then
    run the optimizer on the model's parameters."""

    def __init__(self, model, precision="fp32"):
        if precision not in ("fp32", "bf16"):
            raise ValueError("precision must be 'fp32' or 'bf16'")
        self.precision = precision
        self.mem = getattr(model, "memory_updater", None)
        if precision == "bf16" and self.mem is not None:
            raise NotImplementedError("the bf16 projection mode covers the memoryless attention layers")
        if model.memory_param.get("type", "none") != "none" and self.mem is None:
            raise NotImplementedError("node memory needs memory.MemoryModel")
        self.model = model
        self.last_memory = None
        # APAN (memorys.py:342-385 + layers.py:242-249): the transformer memory
        # updater feeds an identity LayerNorm; no attention layers
        self.apan = model.gnn_param["arch"] == "identity"
        self.mem_kv = _LayerParams.__new__(_LayerParams) if self.apan else None
        if self.apan:
            self.mem_kv.L = self.mem
            self.mem_kv.D = self.mem.dim_out
            self.mem_kv.W_kv = self.mem_kv.b_kv = self.mem_kv.gW_kv = self.mem_kv.gb_kv = None
            self.layers = []
            self.flat = self._build_flat()
            return
        self.layers = [_LayerParams(model.layers["l%dh0" % l]) for l in range(model.gnn_param["layer"])]
        for lp in self.layers:
            if lp.dn + lp.dtime == 0:
                raise NotImplementedError("Q = ones branch (layers.py:137-140) is not on the device path")
            if lp.L.layer_norm.weight.shape[0] % 4 or lp.D % 4:
                raise NotImplementedError("dim_out must be a multiple of 4")
        self.flat = self._build_flat()
        if precision == "bf16":
            self._build_bf16()

    # -- parameter and gradient storage ---------------------------------------
    def _build_flat(self):
        """Re-seats every parameter as a view of one flat buffer (`flat_params`)
        and gives it a .grad view at the same offset of the gradient buffer
        (returned).  w_k / w_v (weights, and biases) become adjacent rows of
        one group, so K and V come from one GEMM."""
        m = self.model
        names = {id(p): n for n, p in m.named_parameters()}
        # Gradient buckets in the order the backward finishes them: the edge
        # predictor with the top layer, then each lower layer, then the
        # memory updater; each bucket is one contiguous range of the buffer,
        # so data-parallel training can all-reduce it while the layers below
        # are still running their backward.
        owners = ["edge_predictor."] + ["layers.l%dh0." % l for l in range(len(self.layers) - 1, -1, -1)]
        groups = []                      # (layer or None, kind, shape, [parameter names], bucket)
        seated = set()

        def bucket_of(name):
            for i, o in enumerate(owners):
                if name.startswith(o):
                    return max(i - 1, 0)          # the predictor shares the top layer's bucket
            return len(owners) - 1

        for lp in self.layers + ([self.mem_kv] if self.apan else []):
            L = lp.L
            bk = bucket_of(names[id(L.w_k.weight)])
            groups.append((lp, "W", (2 * lp.D, L.w_k.weight.shape[1]), [names[id(L.w_k.weight)],
                                                                         names[id(L.w_v.weight)]], bk))
            groups.append((lp, "b", (2 * lp.D,), [names[id(L.w_k.bias)], names[id(L.w_v.bias)]], bk))
            seated.update(id(p) for p in (L.w_k.weight, L.w_v.weight, L.w_k.bias, L.w_v.bias))
        for n_, p in m.named_parameters():
            if id(p) not in seated:
                groups.append((None, None, tuple(p.shape), [n_], bucket_of(n_)))
        groups.sort(key=lambda g: g[4])           # stable: the order within a bucket is kept
        numel = lambda shape: int(torch.Size(shape).numel())
        total = sum((numel(shape) + _ALIGN - 1) // _ALIGN * _ALIGN for _, _, shape, _, _ in groups)
        dev = next(m.parameters()).device
        flat_p = torch.zeros(total, device=dev, dtype=torch.float32)
        flat_g = torch.zeros(total, device=dev, dtype=torch.float32)
        params = dict(m.named_parameters())
        off = 0
        starts = {}
        for lp, kind, shape, members, bk in groups:
            starts.setdefault(bk, off)
            n = numel(shape)
            pv = flat_p[off:off + n].view(shape)
            gv = flat_g[off:off + n].view(shape)
            rows = 0
            for name in members:
                old = params[name]
                r = old.shape[0]
                sl = slice(rows, rows + r) if len(members) > 1 else slice(None)
                pv[sl].copy_(old.data)
                mod_name, attr = name.rsplit(".", 1)
                new = torch.nn.Parameter(pv[sl])
                setattr(m.get_submodule(mod_name), attr, new)
                new.grad = gv[sl]
                rows += r
            if lp is not None:
                if kind == "W":
                    lp.W_kv, lp.gW_kv = pv, gv
                else:
                    lp.b_kv, lp.gb_kv = pv, gv
            off += (n + _ALIGN - 1) // _ALIGN * _ALIGN
        self.flat_params = flat_p
        bks = sorted(starts)
        # (lo, hi) of every bucket, in the order the backward completes them
        self.grad_buckets = [(starts[b], starts[bks[i + 1]] if i + 1 < len(bks) else total)
                             for i, b in enumerate(bks)]
        self._bucket_ids = bks
        return flat_g

    def parameters(self):
        return list(self.model.parameters())

    # -- a second stream for launches nothing downstream waits for ------------
    def _side(self, fn, *uses):
        """Enqueues fn's launches on a side stream, after everything enqueued
        so far on the current stream, so that they overlap the launches that
        follow (a layer's time-encoding and Q-bias gradients run beside the
        next layer's backward).  `uses`: tensors allocated on the current
        stream that fn reads.  The current stream joins the side stream at the
        end of the step (_join); with FB_SIDE_STREAMS=0, fn runs inline."""
        if not SIDE_STREAMS or ops.TIMER is not None:     # the per-kernel timer measures kernels alone
            fn()
            return
        cur = torch.cuda.current_stream()
        if getattr(self, "_side_stream", None) is None or self._side_stream.device != cur.device:
            self._side_stream = torch.cuda.Stream(device=cur.device)
        side = self._side_stream
        side.wait_stream(cur)
        for t in uses:
            if t is not None:
                t.record_stream(side)
        with torch.cuda.stream(side):
            fn()
        self._side_pending = True

    def _side_record(self, fn, *uses):
        """_side, returning an event recorded on the side stream after fn's
        launches (None when fn ran inline): a later launch on the current
        stream that needs fn's results waits on it (_await) instead of on
        the whole side stream."""
        self._side(fn, *uses)
        if not getattr(self, "_side_pending", False) or not SIDE_STREAMS or ops.TIMER is not None:
            return None
        ev = torch.cuda.Event()
        ev.record(self._side_stream)
        return ev

    @staticmethod
    def _await(ev):
        if ev is not None:
            torch.cuda.current_stream().wait_event(ev)

    def _await_weights(self):
        """The current stream waits once per step for the bf16 weight copies."""
        self._await(getattr(self, "_weights_ev", None))
        self._weights_ev = None

    def _in_side(self):
        """Context for launches that must follow everything enqueued so far on
        both streams (a gradient bucket's all-reduce, whose gradients the
        current stream and the side stream wrote): the side stream first
        waits for the current one."""
        import contextlib
        if SIDE_STREAMS and getattr(self, "_side_pending", False):
            self._side_stream.wait_stream(torch.cuda.current_stream())
            return torch.cuda.stream(self._side_stream)
        return contextlib.nullcontext()

    def _join(self):
        if getattr(self, "_side_pending", False):
            torch.cuda.current_stream().wait_stream(self._side_stream)
            self._side_pending = False

    # -- bf16 projection mode -------------------------------------------------
    def _build_bf16(self):
        """bf16 copies of the projection weights in the column layout of the
        bf16 projection rows (segments at multiples of 8, zeros between):
        W_kv over [h | f | time], W_q over [h | time], W_out over [agg | h].
        Refreshed from the fp32 master weights by one cast launch per step."""
        self.cast_jobs = []
        for lp in self.layers:
            L, D, dn, de, dt = lp.L, lp.D, lp.dn, lp.de, lp.dtime
            dev = lp.W_kv.device
            bf = dict(device=dev, dtype=torch.bfloat16)
            (h_at, f_at, t_at), kx = ops.bf16_layout(dn, de, dt)
            lp.kv_segs = [(at, lo, d) for at, lo, d in ((h_at, 0, dn), (f_at, dn, de), (t_at, dn + de, dt)) if d > 0]
            lp.kx = kx
            lp.W_kv_bf = torch.zeros(2 * D, ops.pad8(kx), **bf)
            for at, lo, d in lp.kv_segs:
                self.cast_jobs.append((lp.W_kv[:, lo:lo + d], lp.W_kv_bf[:, at:at + d]))
            if dn > 0:
                (qh, qt), kq = ops.bf16_layout(dn, dt) if dt > 0 else ((0, 0), dn)
                lp.q_segs = [(qh, 0, dn)] + ([(qt, dn, dt)] if dt > 0 else [])
                lp.kq = kq
                lp.W_q_bf = torch.zeros(D, ops.pad8(kq), **bf)
                for at, lo, d in lp.q_segs:
                    self.cast_jobs.append((L.w_q.weight[:, lo:lo + d], lp.W_q_bf[:, at:at + d]))
            # layer 0 reads the feature tables: its projection rows are gathered
            # inside the GEMM (fused_layer0), in 64-column segments [h | f | t]
            lp.g_w = (pad64(dn), pad64(de), pad64(dt))
            if lp is self.layers[0]:
                g_at = (0, lp.g_w[0], lp.g_w[0] + lp.g_w[1])
                lp.g_segs = [(at, lo, d) for at, lo, d in zip(g_at, (0, dn, dn + de), (dn, de, dt)) if d > 0]
                lp.W_kv_g = torch.zeros(2 * D, sum(lp.g_w), **bf)
                for at, lo, d in lp.g_segs:
                    self.cast_jobs.append((lp.W_kv[:, lo:lo + d], lp.W_kv_g[:, at:at + d]))
            lp.ka = ops.pad8(D)
            lp.W_out_bf = torch.zeros(D, ops.pad8(lp.ka + dn), **bf)
            self.cast_jobs.append((L.w_out.weight[:, :D], lp.W_out_bf[:, :D]))
            if dn > 0:
                self.cast_jobs.append((L.w_out.weight[:, D:], lp.W_out_bf[:, lp.ka:lp.ka + dn]))

    def _layer_fwd_bf16(self, l, blk, h, node_table, edge_table, offset_dev, training):
        """_layer_fwd with bf16 projections: bf16 projection rows from the
        gather, K|V, Q and w_out products of bf16 operands accumulated in fp32,
        K|V stored as bf16; attention (fp32 arithmetic), tail and everything
        after in fp32."""
        lp = self.layers[l]
        L, D, dn, de, dtime = lp.L, lp.D, lp.dn, lp.de, lp.dtime
        nd, E = blk.n_dst, blk.n_edges
        nd_dev, E_dev = blk.n_dst_dev, blk.n_edges_dev
        dev = lp.W_kv.device
        if not blk.static and E == 0:
            return None, torch.zeros(nd, D, device=dev)
        wv = L.time_enc.w.weight.view(-1) if dtime > 0 else None
        bt = L.time_enc.w.bias if dtime > 0 else None
        if h is not None:
            if blk.static and not blk.n_dst_static:
                raise NotImplementedError("graph mode feeds a previous layer's output only to the top block")
            hsrc, hdst = dict(h=h, h_off=nd), dict(h=h, h_off=0)
        elif node_table is not None and dn > 0:
            hsrc, hdst = dict(h=node_table, h_idx=blk.src_nodes), dict(h=node_table, h_idx=blk.dst_nodes)
        else:
            hsrc = hdst = {}
        # K|V stored as bf16 rows: the projection's bf16 output is the attention's input
        KV = torch.empty(E, 2 * D, device=dev, dtype=torch.bfloat16)
        gat = self._layer0_gather(l, blk, h, node_table, edge_table, wv, bt, dev)
        P = p_ev = None
        if gat is None and self._node_product(l, h, node_table, E):
            # the node product P = table . W_h^T on the side stream (after the
            # weight cast), beside this layer's gathers
            P = torch.empty(node_table.shape[0], 2 * D, device=dev)
            p_ev = self._side_record(
                lambda: ops.gemm_bf16_group([dict(kind=ops.NT, A=node_table[:, :dn], B=lp.W_kv_bf[:, :dn], out=P)],
                                            name="gemm_group:node_product"), P, node_table)
        if gat is not None:
            # the projection rows [h | f | cos] are gathered inside the GEMM:
            # only the time encoding is written, the tables are read in place
            X = None
            probs = [dict(kind=ops.NT, gather=gat, M=E, B=lp.W_kv_g, bias=lp.b_kv, out=KV, M_dev=E_dev)]
        else:
            X, kx = ops.gather_time_encode_bf16(E, f=edge_table if de > 0 else None, f_idx=blk.eid,
                                                dt=blk.dt_edges, w=wv, b=bt, device=dev, n_rows_dev=E_dev, dn=dn,
                                                de=de, **hsrc)
            probs = [dict(kind=ops.NT, A=X[:, :kx], B=lp.W_kv_bf[:, :kx], bias=lp.b_kv, out=KV, M_dev=E_dev)]
            if P is not None:
                # the node-feature block of every K|V row is the product of one of
                # the table's few rows (P, above); the rows' product runs over their
                # [f | time] columns only and adds P[source node] in its epilogue
                f_at = lp.kv_segs[1][0]
                probs = []
                kv_prob = dict(kind=ops.NT, A=X[:, f_at:kx], B=lp.W_kv_bf[:, f_at:kx], bias=lp.b_kv, out=KV,
                               M_dev=E_dev, add=P, add_idx=blk.src_nodes)
        if dn > 0:
            Qin, kq = ops.gather_time_encode_bf16(nd, w=wv, b=bt, device=dev, n_rows_dev=nd_dev, dn=dn, **hdst)
            Q = torch.empty(nd, D, device=dev)
            probs.append(dict(kind=ops.NT, A=Qin[:, :kq], B=lp.W_q_bf[:, :kq], bias=L.w_q.bias, out=Q, M_dev=nd_dev))
            self._await_weights()
            ops.gemm_bf16_group(probs, name="gemm_group:kv_q")
            if P is not None:
                self._await(p_ev)
                ops.gemm_bf16_group([kv_prob], name="gemm_group:kv_rows")
        else:
            # one shared Q input row cos(b_t): its product stays fp32
            Qin = ops.gather_time_encode(1, w=wv, b=bt, device=dev)
            Q = torch.empty(1, D, device=dev)
            self._await_weights()
            ops.gemm_bf16_group(probs, name="gemm_group:kv_q")
            ops.gemm_group([dict(kind=ops.NT, A=Qin, B=L.w_q.weight, bias=L.w_q.bias, out=Q)], name="gemm_group:q1")
        p_att = L.att_dropout_p if training else 0.0
        # the aggregate is only the w_out product's bf16 operand: written as bf16
        agg_bf = torch.empty(nd, lp.ka, device=dev, dtype=torch.bfloat16)
        att = ops.attn_fwd_kvbf16_bf16out(Q, KV, blk.rptr, L.num_head, L.negative_slope, agg_bf[:, :D], p_att,
                                          0x5EED + l, 0, n_dst_dev=nd_dev, offset_dev=offset_dev)
        agg = None
        Z = torch.empty(nd, D, device=dev)
        if dn > 0:
            p_out = dict(kind=ops.NT, A=agg_bf[:, :D], A2=Qin[:, :dn], k1=lp.ka, B=lp.W_out_bf[:, :lp.ka + dn],
                         bias=L.w_out.bias, out=Z, M_dev=nd_dev)
        else:
            p_out = dict(kind=ops.NT, A=agg_bf[:, :D], B=lp.W_out_bf[:, :D], bias=L.w_out.bias, out=Z, M_dev=nd_dev)
        ops.gemm_bf16_group([p_out], name="gemm_group:w_out")
        p_drop = L.dropout.p if training else 0.0
        y, out = ops.layer_tail_fwd(Z, L.layer_norm.weight, L.layer_norm.bias, eps=L.layer_norm.eps, drop_p=p_drop,
                                    seed=0x7A11 + l, offset_dev=offset_dev, y=Z, n_dev=nd_dev,
                                    gate_dev=E_dev if blk.static else None)
        st = dict(blk=blk, A=X, gather=gat, KV=KV, Qin=Qin, Q=Q, agg=agg, agg_bf=agg_bf, att=att, y=y, p_att=p_att,
                  p_drop=p_drop, offset_dev=offset_dev)
        return st, out

    def _node_product(self, l, h, node_table, E):
        """Layer 0's node-feature product runs per node-table row (then gathered
        by the epilogue) when the table has fewer rows than a quarter of the
        block's edges: bf16 tables read by index, no previous-layer input.
        FB_NODE_PRODUCT=0 keeps the per-edge product."""
        lp = self.layers[l]
        return (NODE_PRODUCT and l == 0 and h is None and lp.dn > 0 and lp.de + lp.dtime > 0 and
                node_table is not None and node_table.dtype == torch.bfloat16 and 4 * node_table.shape[0] < E)

    def _layer0_gather(self, l, blk, h, node_table, edge_table, wv, bt, dev):
        """The gathered projection rows of layer 0 (ops.RowGather), when the
        layer reads bf16 feature tables: node rows by the edges' source node,
        edge rows by edge id, and the time encoding cos(w dt + b), the one
        block written (as [E, pad8(dtime)] bf16).  None: the layer takes the
        previous layer's output, so its rows are materialised."""
        lp = self.layers[l]
        if l != 0 or h is not None or getattr(lp, "W_kv_g", None) is None or FUSED_GATHER_OFF:
            return None
        dn, de, dtime = lp.dn, lp.de, lp.dtime
        if (dn > 0 and (node_table is None or node_table.dtype != torch.bfloat16)) or \
                (de > 0 and (edge_table is None or edge_table.dtype != torch.bfloat16)):
            return None
        segs = []
        if dn > 0:
            segs.append((node_table, dn, blk.src_nodes, lp.g_w[0]))
        if de > 0:
            segs.append((edge_table, de, blk.eid, lp.g_w[1]))
        if dtime > 0:
            T, _ = ops.gather_time_encode_bf16(blk.n_edges, dt=blk.dt_edges, w=wv, b=bt, device=dev,
                                               n_rows_dev=blk.n_edges_dev)
            segs.append((T, dtime, None, lp.g_w[2]))
        return ops.RowGather(segs)

    def _layer_bwd_bf16(self, l, st, dout, dh_rows):
        """_layer_bwd with bf16 operands for every projection-gradient product
        (the gradient rows rounded to bf16: dZ, dK|dV, dQ)."""
        lp = self.layers[l]
        L, D, dn, de, dtime = lp.L, lp.D, lp.dn, lp.de, lp.dtime
        if st is None:
            return None if dh_rows == 0 else torch.zeros(dh_rows, dn, device=dout.device)
        blk = st["blk"]
        nd, E = blk.n_dst, blk.n_edges
        nd_dev, E_dev = blk.n_dst_dev, blk.n_edges_dev
        g = lambda p: p.grad
        dev = dout.device
        dZ = ops.layer_tail_bwd(dout, st["y"], L.layer_norm.weight, g(L.layer_norm.weight), g(L.layer_norm.bias),
                                eps=L.layer_norm.eps, drop_p=st["p_drop"], n_dev=nd_dev,
                                gate_dev=E_dev if blk.static else None)
        dZ_bf = torch.empty(nd, lp.ka, device=dev, dtype=torch.bfloat16)
        ops.cast_bf16([(dZ, dZ_bf[:, :D], nd_dev)])
        dZb = dZ_bf[:, :D]
        gWo = g(L.w_out.weight)
        Qin, agg_bf = st["Qin"], st["agg_bf"]
        dagg = torch.empty(nd, D, device=dev)
        dh = None
        probs = [dict(kind=ops.TN, A=dZb, B=agg_bf[:, :D], out=gWo[:, :D], accumulate=True, M_dev=nd_dev,
                      db=g(L.w_out.bias)),
                 dict(kind=ops.NN, A=dZb, B=lp.W_out_bf[:, :D], out=dagg, M_dev=nd_dev)]
        if dn > 0:
            probs.append(dict(kind=ops.TN, A=dZb, B=Qin[:, :dn], out=gWo[:, D:], accumulate=True, M_dev=nd_dev))
        if dh_rows > 0:
            assert dh_rows >= nd + E
            dh = torch.empty(dh_rows, dn, device=dev)
            probs.append(dict(kind=ops.NN, A=dZb, B=lp.W_out_bf[:, lp.ka:lp.ka + dn], out=dh[:nd], M_dev=nd_dev))
        ops.gemm_bf16_group(probs, name="gemm_group:bwd_dz")
        if dn > 0:
            # dq is only the bf16 operand of the Q-side products: written as bf16
            dQ_bf = torch.empty(nd, lp.ka, device=dev, dtype=torch.bfloat16)
            dKV = ops.attn_bwd_kvbf16_bf16dq(st["Q"], st["KV"], blk.rptr, st["att"], dagg, L.num_head,
                                             L.negative_slope, dQ_bf[:, :D], st["p_att"], 0x5EED + l, 0,
                                             n_dst_dev=nd_dev, offset_dev=st["offset_dev"])
        else:
            dQ, dKV = ops.attn_bwd_kvbf16(st["Q"], st["KV"], blk.rptr, st["att"], dagg, L.num_head,
                                          L.negative_slope, st["p_att"], 0x5EED + l, 0, n_dst_dev=nd_dev,
                                          offset_dev=st["offset_dev"])
        X, gat = st["A"], st["gather"]
        v = torch.empty(D, device=dev)            # sum over rows of dQ
        # the K|V weight and bias gradient over the whole projection row: one
        # TN problem, X's segments mapped to the weight's columns (gathered
        # rows: the same segments read from the tables again)
        if gat is not None:
            probs = [dict(kind=ops.TN, A=dKV, gather=gat, out=lp.gW_kv, accumulate=True, M_dev=E_dev,
                          db=lp.gb_kv, segs=[(at, d, lo) for at, lo, d in lp.g_segs])]
            W_t, t_at = lp.W_kv_g, lp.g_segs[-1][0]
        else:
            probs = [dict(kind=ops.TN, A=dKV, B=X[:, :lp.kx], out=lp.gW_kv, accumulate=True, M_dev=E_dev,
                          db=lp.gb_kv, segs=[(at, d, lo) for at, lo, d in lp.kv_segs])]
            W_t, t_at = lp.W_kv_bf, lp.kv_segs[-1][0]
        if dh is not None:
            probs.append(dict(kind=ops.NN, A=dKV, B=lp.W_kv_bf[:, :dn], out=dh[nd:nd + E], M_dev=E_dev))
        dA_t = None
        if dtime > 0:
            # bf16, like the gradient of an autocast bf16 product; summed in fp32
            # rows padded to 16 bytes: the bf16 product stores measured up to 4x slower on 200-byte rows
            dA_t = torch.empty(E, ops.pad8(dtime), device=dev, dtype=torch.bfloat16)[:, :dtime]
            probs.append(dict(kind=ops.NN, A=dKV, B=W_t[:, t_at:t_at + dtime], out=dA_t, M_dev=E_dev))
        if dn > 0:
            dQb = dQ_bf[:, :D]
            probs.append(dict(kind=ops.TN, A=dQb, B=Qin[:, :lp.kq], out=g(L.w_q.weight), accumulate=True,
                              M_dev=nd_dev, db=v, db_accumulate=False, segs=[(at, d, lo) for at, lo, d in lp.q_segs]))
            if dh is not None:
                probs.append(dict(kind=ops.NN, A=dQb, B=lp.W_q_bf[:, :dn], out=dh[:nd], accumulate=True,
                                  M_dev=nd_dev))
            ops.gemm_bf16_group(probs, name="gemm_group:bwd_dkv_dq")
        else:
            ops.gemm_bf16_group(probs, name="gemm_group:bwd_dkv_dq")
            ops.gemm_group([dict(kind=ops.TN, A=dQ, B=None, out=None, M_dev=nd_dev, db=v, db_accumulate=False)],
                           name="gemm_group:dq_sum")
        self._side(lambda: self._time_grads(l, st, dA_t, v), dA_t, v, st["Qin"])
        return dh

    def _time_grads(self, l, st, dA_t, v):
        """The time encoder's and the Q bias's gradients of layer l, from the
        time-encoding input gradient dA_t and v = sum over rows of dQ: nothing
        else in the step reads them."""
        lp = self.layers[l]
        L, dn, dtime = lp.L, lp.dn, lp.dtime
        blk = st["blk"]
        g = lambda p: p.grad
        if dtime > 0:
            ops.time_encode_bwd(dA_t, blk.dt_edges, L.time_enc.w.weight.view(-1), L.time_enc.w.bias,
                                g(L.time_enc.w.weight).view(-1), g(L.time_enc.w.bias), n_dev=blk.n_edges_dev)
        bt = L.time_enc.w.bias if dtime > 0 else None
        gbt = g(L.time_enc.w.bias) if dtime > 0 else None
        if dn == 0:
            # one shared Q input row cos(b_t): every Q-side gradient needs only sum_rows dQ
            ops.q_time_bwd(v, L.w_q.weight, dn, dtime, bt, g(L.w_q.bias), gbt, qin0=st["Qin"][0],
                           dW_q=g(L.w_q.weight))
        else:
            ops.q_time_bwd(v, L.w_q.weight, dn, dtime, bt, g(L.w_q.bias), gbt)

    # -- one layer ------------------------------------------------------------
    def _layer_fwd(self, l, blk, h, node_table, edge_table, offset_dev, training):
        lp = self.layers[l]
        L, D, dn, de, dtime = lp.L, lp.D, lp.dn, lp.de, lp.dtime
        nd, E = blk.n_dst, blk.n_edges
        nd_dev, E_dev = blk.n_dst_dev, blk.n_edges_dev
        dev = lp.W_kv.device
        if not blk.static and E == 0:
            # layers.py:101-102: a block without edges outputs zeros
            return None, torch.zeros(nd, D, device=dev)
        wv = L.time_enc.w.weight.view(-1) if dtime > 0 else None
        bt = L.time_enc.w.bias if dtime > 0 else None
        if h is not None:
            if blk.static and not blk.n_dst_static:
                raise NotImplementedError("graph mode feeds a previous layer's output only to the top block")
            hsrc, hdst = dict(h=h, h_off=nd), dict(h=h, h_off=0)
        elif node_table is not None and dn > 0:
            hsrc, hdst = dict(h=node_table, h_idx=blk.src_nodes), dict(h=node_table, h_idx=blk.dst_nodes)
        else:
            hsrc = hdst = {}
        A = ops.gather_time_encode(E, f=edge_table if de > 0 else None, f_idx=blk.eid, dt=blk.dt_edges, w=wv, b=bt,
                                   device=dev, n_rows_dev=E_dev, **hsrc)
        if dn > 0:
            Qin = ops.gather_time_encode(nd, w=wv, b=bt, device=dev, n_rows_dev=nd_dev, **hdst)
        else:
            Qin = ops.gather_time_encode(1, w=wv, b=bt, device=dev)
        KV = torch.empty(E, 2 * D, device=dev)
        Q = torch.empty(Qin.shape[0], D, device=dev)
        ops.gemm_group([dict(kind=ops.NT, A=A, B=lp.W_kv, bias=lp.b_kv, out=KV, M_dev=E_dev),
                        dict(kind=ops.NT, A=Qin, B=L.w_q.weight, bias=L.w_q.bias, out=Q,
                             M_dev=nd_dev if dn > 0 else None)], name="gemm_group:kv_q")
        p_att = L.att_dropout_p if training else 0.0
        agg, att = ops.attn_fwd(Q, KV[:, :D], KV[:, D:], blk.rptr, L.num_head, L.negative_slope, p_att,
                                0x5EED + l, 0, n_dst_dev=nd_dev, offset_dev=offset_dev)
        # w_out([agg | h_dst]) as one GEMM over the concatenation along K (h_dst = Qin[:, :dn])
        Z = torch.empty(nd, D, device=dev)
        ops.gemm_group([dict(kind=ops.NT, A=agg, A2=Qin[:, :dn] if dn > 0 else None, B=L.w_out.weight,
                             bias=L.w_out.bias, out=Z, M_dev=nd_dev)], name="gemm_group:w_out")
        p_drop = L.dropout.p if training else 0.0
        y, out = ops.layer_tail_fwd(Z, L.layer_norm.weight, L.layer_norm.bias, eps=L.layer_norm.eps, drop_p=p_drop,
                                    seed=0x7A11 + l, offset_dev=offset_dev, y=Z, n_dev=nd_dev,
                                    gate_dev=E_dev if blk.static else None)
        st = dict(blk=blk, A=A, KV=KV, Qin=Qin, Q=Q, agg=agg, att=att, y=y, p_att=p_att, p_drop=p_drop,
                  offset_dev=offset_dev)
        return st, out

    def _layer_bwd(self, l, st, dout, dh_rows):
        """Adds layer l's parameter gradients; returns the gradient of its
        input h (dh_rows rows: the layer below's destinations, or for layer 0 of
        a memory model its source rows), or None when dh_rows == 0."""
        lp = self.layers[l]
        L, D, dn, de, dtime = lp.L, lp.D, lp.dn, lp.de, lp.dtime
        if st is None:                     # empty block (eager): zero output, no gradient
            return None if dh_rows == 0 else torch.zeros(dh_rows, dn, device=dout.device)
        blk = st["blk"]
        nd, E = blk.n_dst, blk.n_edges
        nd_dev, E_dev = blk.n_dst_dev, blk.n_edges_dev
        g = lambda p: p.grad
        dZ = ops.layer_tail_bwd(dout, st["y"], L.layer_norm.weight, g(L.layer_norm.weight), g(L.layer_norm.bias),
                                eps=L.layer_norm.eps, drop_p=st["p_drop"], n_dev=nd_dev,
                                gate_dev=E_dev if blk.static else None)
        Wo, gWo = L.w_out.weight, g(L.w_out.weight)
        agg, Qin = st["agg"], st["Qin"]
        dev = dout.device
        dagg = torch.empty(nd, D, device=dev)
        dh = None
        # every product that reads dZ, in one launch
        probs = [dict(kind=ops.TN, A=dZ, B=agg, out=gWo[:, :D], accumulate=True, M_dev=nd_dev, db=g(L.w_out.bias)),
                 dict(kind=ops.NN, A=dZ, B=Wo[:, :D], out=dagg, M_dev=nd_dev)]
        if dn > 0:
            probs.append(dict(kind=ops.TN, A=dZ, B=Qin[:, :dn], out=gWo[:, D:], accumulate=True, M_dev=nd_dev))
        if dh_rows > 0:                    # the layer's input h needs a gradient (layer above, or the memory)
            assert dh_rows >= nd + E
            dh = torch.empty(dh_rows, dn, device=dev)
            probs.append(dict(kind=ops.NN, A=dZ, B=Wo[:, D:], out=dh[:nd], M_dev=nd_dev))
        ops.gemm_group(probs, name="gemm_group:bwd_dz")
        KV = st["KV"]
        dQ, dKV = ops.attn_bwd(st["Q"], KV[:, :D], KV[:, D:], blk.rptr, st["att"], dagg, L.num_head,
                               L.negative_slope, st["p_att"], 0x5EED + l, 0, n_dst_dev=nd_dev,
                               offset_dev=st["offset_dev"])
        # every product that reads dKV or dQ, in one launch
        v = torch.empty(D, device=dev)            # sum over rows of dQ
        probs = [dict(kind=ops.TN, A=dKV, B=st["A"], out=lp.gW_kv, accumulate=True, M_dev=E_dev, db=lp.gb_kv)]
        if dh is not None:
            probs.append(dict(kind=ops.NN, A=dKV, B=lp.W_kv[:, :dn], out=dh[nd:nd + E], M_dev=E_dev))
        dA_t = None
        if dtime > 0:
            dA_t = torch.empty(E, dtime, device=dev)
            probs.append(dict(kind=ops.NN, A=dKV, B=lp.W_kv[:, dn + de:], out=dA_t, M_dev=E_dev))
        if dn == 0:
            probs.append(dict(kind=ops.TN, A=dQ, B=None, out=None, M_dev=nd_dev, db=v, db_accumulate=False))
        else:
            probs.append(dict(kind=ops.TN, A=dQ, B=Qin, out=g(L.w_q.weight), accumulate=True, M_dev=nd_dev,
                              db=v, db_accumulate=False))
            if dh is not None:
                probs.append(dict(kind=ops.NN, A=dQ, B=L.w_q.weight[:, :dn], out=dh[:nd], accumulate=True,
                                  M_dev=nd_dev))
        ops.gemm_group(probs, name="gemm_group:bwd_dkv_dq")
        self._side(lambda: self._time_grads(l, st, dA_t, v), dA_t, v, Qin)
        return dh

    # -- node memory (GRU updater) ---------------------------------------------
    def _memory_fwd(self, blk, mailbox):
        """h' = GRUCell([mail | time encoding], memory) for the source rows of
        blk (memorys.py:284-304); returns h' [n_src, dim_mem] and the saved
        state for the backward."""
        U = self.mem
        cell = U.updater
        H = U.dim_hid
        n, n_dev = blk.n_src, blk.n_src_dev
        dev = cell.weight_ih.device
        din = cell.weight_ih.shape[1]
        x = torch.empty(n, din, device=dev)
        h0 = torch.empty(n, H, device=dev)
        dtm = torch.empty(n, device=dev)
        mailbox.gather(blk.nodes, blk.ts, n, n_dev, U.time_enc if U.dim_time > 0 else None, x, h0, dtm)
        gi = torch.empty(n, 3 * H, device=dev)
        gh = torch.empty(n, 3 * H, device=dev)
        ops.gemm_group([dict(kind=ops.NT, A=x, B=cell.weight_ih, bias=cell.bias_ih, out=gi, M_dev=n_dev),
                        dict(kind=ops.NT, A=h0, B=cell.weight_hh, bias=cell.bias_hh, out=gh, M_dev=n_dev)],
                       name="gemm_group:gru")
        h1 = torch.empty(n, H, device=dev)
        ops.gru_fwd(gi, gh, h0, h1, n_dev=n_dev)
        return h1, dict(x=x, h0=h0, dtm=dtm, gi=gi, gh=gh, n=n, n_dev=n_dev)

    def _memory_bwd(self, st, dh1):
        U = self.mem
        cell = U.updater
        g = lambda p: p.grad
        ops.gru_bwd(st["gi"], st["gh"], st["h0"], dh1, n_dev=st["n_dev"])
        dgi, dgh, n_dev = st["gi"], st["gh"], st["n_dev"]
        dmail = cell.weight_ih.shape[1] - U.dim_time
        probs = [dict(kind=ops.TN, A=dgi, B=st["x"], out=g(cell.weight_ih), accumulate=True, M_dev=n_dev,
                      db=g(cell.bias_ih)),
                 dict(kind=ops.TN, A=dgh, B=st["h0"], out=g(cell.weight_hh), accumulate=True, M_dev=n_dev,
                      db=g(cell.bias_hh))]
        dxt = None
        if U.dim_time > 0:
            dxt = torch.empty(st["n"], U.dim_time, device=dgi.device)
            probs.append(dict(kind=ops.NN, A=dgi, B=cell.weight_ih[:, dmail:], out=dxt, M_dev=n_dev))
        ops.gemm_group(probs, name="gemm_group:gru_bwd")
        if dxt is not None:
            te = U.time_enc
            ops.time_encode_bwd(dxt, st["dtm"], te.w.weight.view(-1), te.w.bias, g(te.w.weight).view(-1),
                                g(te.w.bias), n_dev=n_dev)

    # -- APAN: transformer memory updater + identity LayerNorm -----------------
    def _apan_step(self, roots, root_ts, mailbox, loss_out, scores, training, offset_dev):
        """TransformerMemoryUpdater.forward (memorys.py:358-385) on all roots,
        IdentityNormLayer (layers.py:248-249), edge predictor, loss, and the
        backward of all of it."""
        U, m = self.mem, self.model
        g = lambda p: p.grad
        dev = self.flat.device
        n = roots.shape[0]
        S, D, H = mailbox.size, U.dim_out, U.att_h
        dmail = mailbox.dim_mail
        kin = dmail + U.dim_time
        x = torch.empty(n * S, kin, device=dev)
        h0 = torch.empty(n, D, device=dev)
        dts = torch.empty(n * S, device=dev)
        mailbox.gather_slots(roots, root_ts, n, None, U.time_enc if U.dim_time > 0 else None, x, h0, dts)
        kvp = self.mem_kv
        KV = torch.empty(n * S, 2 * D, device=dev)
        Q = torch.empty(n, D, device=dev)
        ops.gemm_group([dict(kind=ops.NT, A=x, B=kvp.W_kv, bias=kvp.b_kv, out=KV),
                        dict(kind=ops.NT, A=h0, B=U.w_q.weight, bias=U.w_q.bias, out=Q)], name="gemm_group:kv_q")
        rptr = torch.arange(0, n * S + 1, S, dtype=torch.int32, device=dev)   # every root: its S slots
        p_att = U.att_dropout_p if training else 0.0
        agg, att = ops.attn_fwd(Q, KV[:, :D], KV[:, D:], rptr, H, U.negative_slope, p_att, 0x5EED + 9, 0,
                                offset_dev=offset_dev)
        ln1, xhat1, rstd1 = ops.add_layernorm_fwd(agg, h0, U.layer_norm.weight, U.layer_norm.bias,
                                                  eps=U.layer_norm.eps)
        Z = torch.empty(n, D, device=dev)
        ops.gemm_group([dict(kind=ops.NT, A=ln1, B=U.mlp.weight, bias=U.mlp.bias, out=Z)], name="gemm_group:w_out")
        norm = m.layers["l0h0"].norm
        p_drop = U.dropout.p if training else 0.0
        # y = relu(dropout(mlp(.))) is the updated memory; out = the identity layer's LayerNorm of it
        y, out = ops.layer_tail_fwd(Z, norm.weight, norm.bias, eps=norm.eps, drop_p=p_drop, seed=0x7A11 + 9,
                                    offset_dev=offset_dev, y=Z)
        self.last_memory = y
        dh = self._predictor(out, loss_out, scores)
        # backward
        dZ = ops.layer_tail_bwd(dh, y, norm.weight, g(norm.weight), g(norm.bias), eps=norm.eps, drop_p=p_drop)
        dln1 = torch.empty(n, D, device=dev)
        ops.gemm_group([dict(kind=ops.TN, A=dZ, B=ln1, out=g(U.mlp.weight), accumulate=True, db=g(U.mlp.bias)),
                        dict(kind=ops.NN, A=dZ, B=U.mlp.weight, out=dln1)], name="gemm_group:bwd_dz")
        dagg = ops.add_layernorm_bwd(dln1, xhat1, rstd1, U.layer_norm.weight, g(U.layer_norm.weight),
                                     g(U.layer_norm.bias))
        dQ, dKV = ops.attn_bwd(Q, KV[:, :D], KV[:, D:], rptr, att, dagg, H, U.negative_slope, p_att, 0x5EED + 9, 0,
                               offset_dev=offset_dev)
        probs = [dict(kind=ops.TN, A=dKV, B=x, out=kvp.gW_kv, accumulate=True, db=kvp.gb_kv),
                 dict(kind=ops.TN, A=dQ, B=h0, out=g(U.w_q.weight), accumulate=True, db=g(U.w_q.bias))]
        dxt = None
        if U.dim_time > 0:
            dxt = torch.empty(n * S, U.dim_time, device=dev)
            probs.append(dict(kind=ops.NN, A=dKV, B=kvp.W_kv[:, dmail:], out=dxt))
        ops.gemm_group(probs, name="gemm_group:bwd_dkv_dq")
        if dxt is not None:
            te = U.time_enc
            ops.time_encode_bwd(dxt, dts, te.w.weight.view(-1), te.w.bias, g(te.w.weight).view(-1), g(te.w.bias))
        return loss_out

    def _predictor(self, h, loss_out, scores):
        """EdgePredictor + BCE loss forward and backward; returns dh."""
        ep = self.model.edge_predictor
        dev = h.device
        B = h.shape[0] // 3
        D = h.shape[1]
        S = torch.empty(B, D, device=dev)
        P = torch.empty(2 * B, D, device=dev)
        ops.gemm_group([dict(kind=ops.NT, A=h[:B], B=ep.src_fc.weight, bias=ep.src_fc.bias, out=S),
                        dict(kind=ops.NT, A=h[B:3 * B], B=ep.dst_fc.weight, bias=ep.dst_fc.bias, out=P)],
                       name="gemm_group:pred")
        dS = torch.empty(B, D, device=dev)
        dP = torch.empty(2 * B, D, device=dev)
        ops.edge_predictor_loss(S, P, ep.out_fc.weight.view(-1), ep.out_fc.bias, loss_out, dS, dP,
                                ep.out_fc.weight.grad.view(-1), ep.out_fc.bias.grad, scores=scores)
        dh = torch.empty(3 * B, D, device=dev)
        ops.gemm_group([
            dict(kind=ops.TN, A=dS, B=h[:B], out=ep.src_fc.weight.grad, accumulate=True, db=ep.src_fc.bias.grad),
            dict(kind=ops.TN, A=dP, B=h[B:3 * B], out=ep.dst_fc.weight.grad, accumulate=True,
                 db=ep.dst_fc.bias.grad),
            dict(kind=ops.NN, A=dS, B=ep.src_fc.weight, out=dh[:B]),
            dict(kind=ops.NN, A=dP, B=ep.dst_fc.weight, out=dh[B:3 * B])], name="gemm_group:pred_bwd")
        return dh

    # -- whole step -----------------------------------------------------------
    def _buckets_done(self, hook, upto):
        """Calls hook(i) for every gradient bucket i < upto not yet reported
        (on the side stream when side launches wrote into it)."""
        if hook is None:
            return
        with self._in_side():
            while self._reported < min(upto, len(self.grad_buckets)):
                hook(self._reported)
                self._reported += 1

    def step(self, blocks, node_table, edge_table, loss_out, zero_grad=True, scores=None, mailbox=None,
             roots=None, root_ts=None, grad_hook=None):
        """blocks in sampler order (hop 1 first), Device- or StaticBlocks.
        Writes the loss into loss_out (a 0-d device tensor) and the gradients
        into the parameters' .grad (zeroed first unless zero_grad=False);
        with `scores` ([2B] device tensor) also the positive then negative
        edge scores.  Memory models read their inputs from `mailbox` and
        leave the updated memory of the first layer's source rows in
        `last_memory`; APAN models take the batch's roots and times (its
        updater runs on the roots, not on the sampled block).
        grad_hook(i), when given, is called (on the host, in stream order) as
        soon as the launches that write gradient bucket i
        (self.grad_buckets[i], a range of self.flat) are enqueued: the
        predictor's and the top layer's after that layer's backward, each
        lower layer's after its own, every bucket by the end of the call."""
        self._reported = 0
        m = self.model
        training = m.training
        mfgs = list(reversed(blocks))
        dev = self.flat.device
        if m._drop_step is None or m._drop_step.device != dev:
            m._drop_step = torch.zeros(1, dtype=torch.int64, device=dev)
        if training:
            m._drop_step += 1
        if zero_grad:
            self.flat.zero_()
        if self.apan:
            if mailbox is None or roots is None:
                raise ValueError("an APAN step needs its MailBox and the batch's roots")
            out = self._apan_step(roots, root_ts, mailbox, loss_out, scores, training, m._drop_step)
            self._buckets_done(grad_hook, len(self.grad_buckets))
            return out
        saved, h = [], None
        mem_st = None
        if self.mem is not None:
            if mailbox is None:
                raise ValueError("a memory model needs its MailBox")
            h, mem_st = self._memory_fwd(mfgs[0], mailbox)
            self.last_memory = h
        bf16 = self.precision == "bf16"
        self._weights_ev = None
        if bf16:
            # the bf16 weight copies on the side stream, beside layer 0's gathers;
            # the first product that reads them waits for them
            self._weights_ev = self._side_record(lambda: ops.cast_bf16(self.cast_jobs, name="cast_bf16:weights"))
        fwd = self._layer_fwd_bf16 if bf16 else self._layer_fwd
        bwd = self._layer_bwd_bf16 if bf16 else self._layer_bwd
        for l, blk in enumerate(mfgs):
            st, h = fwd(l, blk, h, node_table if (l == 0 and mem_st is None) else None, edge_table,
                        m._drop_step, training)
            saved.append(st)
        dh = self._predictor(h, loss_out, scores)
        n_layers = len(mfgs)
        for l in range(n_layers - 1, -1, -1):
            rows = mfgs[l - 1].n_dst if l > 0 else (mfgs[0].n_src if mem_st is not None else 0)
            dh = bwd(l, saved[l], dh, rows)
            # bucket b holds layer n_layers - 1 - b (bucket 0 also the predictor)
            self._buckets_done(grad_hook, n_layers - l)
        if mem_st is not None:
            if dh is None:                   # an empty block: no gradient reaches the memory updater
                dh = torch.zeros(mem_st["n"], self.mem.dim_hid, device=dev)
            self._memory_bwd(mem_st, dh)
        self._buckets_done(grad_hook, len(self.grad_buckets))
        self._join()
        return loss_out


class FlatAdam:
    """torch.optim.Adam (betas, eps; no weight decay, as the reference's
    train.py:128 uses it) over FusedStep's flat parameter and gradient
    buffers: one kernel per step, the step count on the device (CUDA-graph
    safe)."""

    def __init__(self, engine, lr, betas=(0.9, 0.999), eps=1e-8):
        self.p, self.g = engine.flat_params, engine.flat
        self.m = torch.zeros_like(self.p)
        self.v = torch.zeros_like(self.p)
        self.t = torch.zeros(1, dtype=torch.int64, device=self.p.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.p.device)
        self.lr, self.betas, self.eps = float(lr), betas, float(eps)

    def step(self):
        from .capi import call, ptr, stream_ptr
        ops._launch("adam", 4 * 7 * self.p.numel(), 0, 1,
                    lambda: call("fb_adam_step", ptr(self.p), ptr(self.g), ptr(self.m), ptr(self.v), self.p.numel(),
                                 self.lr, float(self.betas[0]), float(self.betas[1]), self.eps, ptr(self.t),
                                 ptr(self.done), stream_ptr()))

    def zero_grad(self, set_to_none=False):
        self.g.zero_()
