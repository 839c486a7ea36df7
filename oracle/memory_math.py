"""TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference's TGN node
memory (memorys.py) for the parity tests.

Only tests/ use this module, as the checker.  It restates, in the dtype of
the module passed in (fp32 or fp64):
  MailBox.prep_input_mails          memorys.py:51-73
  GRUMemeoryUpdater.forward         memorys.py:284-304 (torch.nn.GRUCell's
                                    documented equations, written out)
  GeneralModel.forward with memory  modules.py:48-70
  MailBox.update_mailbox 'self'     memorys.py:101-142
  MailBox.update_memory             memorys.py:84-99
  TransformerMemoryUpdater.forward  memorys.py:358-385 (APAN)
  IdentityNormLayer                 layers.py:242-249
  MailBox.update_mailbox 'neighbors' memorys.py:143-178 (APAN)
Index assignments with repeated node ids keep the last occurrence, which is
what the reference's CPU tensors do; the loops below write in list order.
"""
import numpy as np
import torch

from .ref_math import layer_forward, time_encode


class MemoryState:
    """The MailBox tables (memorys.py:13-19) as CPU tensors."""

    def __init__(self, num_nodes, dim_mem, dim_edge, mailbox_size=1, dtype=torch.float32):
        self.node_memory = torch.zeros(num_nodes, dim_mem, dtype=dtype)
        self.node_memory_ts = torch.zeros(num_nodes, dtype=torch.float32)
        self.mailbox = torch.zeros(num_nodes, mailbox_size, 2 * dim_mem + dim_edge, dtype=dtype)
        self.mailbox_ts = torch.zeros(num_nodes, mailbox_size, dtype=torch.float32)
        self.next_mail_pos = torch.zeros(num_nodes, dtype=torch.long)
        self.size = mailbox_size


def gru_cell(cell, x, h):
    """torch.nn.GRUCell: r = s(W_ir x + b_ir + W_hr h + b_hr),
    z = s(W_iz x + b_iz + W_hz h + b_hz), n = tanh(W_in x + b_in + r (W_hn h + b_hn)),
    h' = (1 - z) n + z h."""
    gi = torch.nn.functional.linear(x, cell.weight_ih, cell.bias_ih)
    gh = torch.nn.functional.linear(h, cell.weight_hh, cell.bias_hh)
    i_r, i_z, i_n = gi.chunk(3, 1)
    h_r, h_z, h_n = gh.chunk(3, 1)
    r = torch.sigmoid(i_r + h_r)
    z = torch.sigmoid(i_z + h_z)
    n = torch.tanh(i_n + r * h_n)
    return (1 - z) * n + z * h


def memory_forward(updater, state, nodes, ts):
    """prep_input_mails + GRUMemeoryUpdater.forward for a block's source rows
    (nodes, ts: numpy); returns the updated memory [n_src, dim_mem]."""
    idx = torch.from_numpy(np.asarray(nodes)).long()
    dty = updater.updater.weight_ih.dtype
    mem = state.node_memory[idx].to(dty)
    mem_ts = state.node_memory_ts[idx]
    mail = state.mailbox[idx].reshape(idx.shape[0], -1).to(dty)
    x = mail
    if updater.dim_time > 0:
        dt = torch.from_numpy(np.asarray(ts)).float() - mem_ts
        x = torch.cat([mail, time_encode(updater.time_enc, dt)], dim=1)
    return gru_cell(updater.updater, x, mem)


def model_forward(model, state, block, edge_feats, neg_samples=1):
    """GeneralModel.forward with node memory and one attention layer; block
    has row()/col()/eid()/dts()/nodes()/ts()/dim_out() numpy accessors.
    Returns (pred_pos, pred_neg, updated memory of the source rows)."""
    layer = model.layers["l0h0"]
    h = memory_forward(model.memory_updater, state, block.nodes(), block.ts())
    n_dst = int(block.dim_out())
    row = torch.from_numpy(block.row())
    col = torch.from_numpy(block.col())
    dt = torch.from_numpy(block.dts())[n_dst:]
    f = edge_feats[torch.from_numpy(block.eid()).long()].to(h.dtype) if layer.dim_edge_feat > 0 else None
    out = layer_forward(layer, row, col, dt, n_dst, h=h, f=f)
    pos, neg = model.edge_predictor(out, neg_samples=neg_samples)
    return pos, neg, h


def update_mailbox_self(state, roots, root_ts, h, batch_edge_feats):
    """update_mailbox, deliver_to 'self', mail_combine 'last': entry 2i is
    the src of positive edge i with mail [h_src | h_dst | f_i], entry 2i + 1
    its dst with [h_dst | h_src | f_i]; the mail time of entry k is
    root_ts[k] (the reference slices ts[:2n] with the interleaved k)."""
    n = len(roots) // 3
    h = h.detach()
    for k in range(2 * n):
        i = k // 2
        a, b = (i, n + i) if k % 2 == 0 else (n + i, i)
        node = int(roots[a])
        parts = [h[a], h[b]]
        if batch_edge_feats is not None:
            parts.append(batch_edge_feats[i].to(h.dtype))
        pos = int(state.next_mail_pos[node])
        state.mailbox[node, pos] = torch.cat(parts).to(state.mailbox.dtype)
        state.mailbox_ts[node, pos] = float(root_ts[k])
    if state.size > 1:
        for node in set(int(r) for r in roots[:2 * n]):
            state.next_mail_pos[node] = (state.next_mail_pos[node] + 1) % state.size


def update_memory(state, roots, root_ts, h):
    """update_memory: node_memory[roots[k]] = h[k], node_memory_ts[roots[k]] =
    root_ts[k] for k < 2n, in list order."""
    n = len(roots) // 3
    h = h.detach()
    for k in range(2 * n):
        node = int(roots[k])
        state.node_memory[node] = h[k].to(state.node_memory.dtype)
        state.node_memory_ts[node] = float(root_ts[k])


def transformer_memory_forward(U, state, roots, ts):
    """TransformerMemoryUpdater.forward (memorys.py:358-385) for the roots
    (node_to_dgl_blocks: no sampled neighbours); returns the updated memory."""
    idx = torch.from_numpy(np.asarray(roots)).long()
    dty = U.w_q.weight.dtype
    n = idx.shape[0]
    S = state.size
    mem = state.node_memory[idx].to(dty)
    mail = state.mailbox[idx].to(dty)                      # [n, S, dmail]
    H = U.att_h
    Q = U.w_q(mem).reshape(n, H, -1)
    if U.dim_time > 0:
        dt = torch.from_numpy(np.asarray(ts)).float()[:, None] - state.mailbox_ts[idx]
        tf = time_encode(U.time_enc, dt.reshape(-1)).reshape(n, S, -1)
        mail = torch.cat([mail, tf], dim=2)
    K = U.w_k(mail).reshape(n, S, H, -1)
    V = U.w_v(mail).reshape(n, S, H, -1)
    att = torch.nn.functional.leaky_relu((Q[:, None, :, :] * K).sum(dim=3), 0.2)
    att = torch.softmax(att, dim=1)
    rst = (att[:, :, :, None] * V).sum(dim=1).reshape(n, -1)
    rst = rst + mem
    rst = U.layer_norm(rst)
    rst = U.mlp(rst)
    rst = U.dropout(rst)
    return torch.relu(rst)


def apan_forward(model, state, roots, ts, neg_samples=1):
    """GeneralModel.forward of APAN: memory updater on the roots, the identity
    layer's LayerNorm, edge predictor.  Returns (pred_pos, pred_neg, updated
    memory)."""
    h = transformer_memory_forward(model.memory_updater, state, roots, ts)
    out = model.layers["l0h0"].norm(h)
    pos, neg = model.edge_predictor(out, neg_samples=neg_samples)
    return pos, neg, h


def update_mailbox_neighbors(state, roots, root_ts, h, batch_edge_feats, block_nodes, block_row):
    """update_mailbox, deliver_to 'neighbors', mail_combine 'last': the mail of
    positive root j is [h_j | h_other | f_i] (src roots j < n, then dst roots),
    its time root_ts[j]; list entry k < 2n is root k itself, entry 2n + e the
    node sampled for edge e, which gets the mail of its root row[e].  Each
    node keeps its last entry, written to its next slot, which then advances."""
    n = len(roots) // 3
    h = h.detach()
    last = {}
    for k, node in enumerate(np.asarray(block_nodes)):
        last[int(node)] = k
    for node, k in last.items():
        j = k if k < 2 * n else int(block_row[k - 2 * n])
        other, ei = (j + n, j) if j < n else (j - n, j - n)
        parts = [h[j], h[other]]
        if batch_edge_feats is not None:
            parts.append(batch_edge_feats[ei].to(h.dtype))
        pos = int(state.next_mail_pos[node])
        state.mailbox[node, pos] = torch.cat(parts).to(state.mailbox.dtype)
        state.mailbox_ts[node, pos] = float(root_ts[j])
        if state.size > 1:
            state.next_mail_pos[node] = (pos + 1) % state.size
