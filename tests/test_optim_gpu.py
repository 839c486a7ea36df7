"""GPU: FlatAdam (one kernel over FusedStep's flat parameter/gradient
buffers, device step count) takes the same steps as torch.optim.Adam on the
same model, and keeps taking them when replayed inside a CUDA graph."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    from fast_b200.model import GeneralModel
    sp = dict(layer=2, neighbor=[10, 10], strategy="recent", prop_time=False, history=1, duration=0)
    gp = dict(arch="transformer_attention", layer=2, att_head=2, dim_time=100, dim_out=100)
    torch.manual_seed(0)
    return GeneralModel(0, 48, sp, dict(type="none", dim_out=0), gp, dict(lr=1e-3, dropout=0.0, att_dropout=0.0))


def test_flat_adam_matches_torch_adam(cuda):
    from fast_b200.engine import FlatAdam, FusedStep
    ref = _model().to(cuda)
    mine = _model().to(cuda)
    eng = FusedStep(mine)
    opt = FlatAdam(eng, 1e-3)
    topt = torch.optim.Adam(ref.parameters(), lr=1e-3)
    g = torch.Generator(device=cuda).manual_seed(1)
    graph = None
    for step in range(8):
        grads = [torch.randn(p.shape, device=cuda, generator=g) * (10.0 ** (step % 3 - 1)) for p in ref.parameters()]
        for p, gr in zip(ref.parameters(), grads):
            p.grad = gr.clone()
        for p, gr in zip(mine.parameters(), grads):
            p.grad.copy_(gr)
        topt.step()
        if step < 4:
            opt.step()
        else:                                   # steps 4.. replay a captured optimizer step
            if graph is None:
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    opt.step()
            graph.replay()
        for (n, pr), pm in zip(ref.named_parameters(), mine.parameters()):
            torch.testing.assert_close(pm, pr, rtol=1e-5, atol=1e-7, msg=lambda m: "step %d %s: %s" % (step, n, m))
    assert int(opt.t.item()) == 8
