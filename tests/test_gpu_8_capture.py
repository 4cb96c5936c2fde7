"""The drop-in contract of basal's graph engine (basal/gemma4_graph.py:96-107, :296: layer functions compiled by
torch.compile with Inductor; basal/engine.py:2273-2307: the forwards captured in CUDA graphs and replayed on new
inputs copied into static buffers) holds for this build's ops:

  - a layer function calling lean.linear with the FP8-block, INT8-block and NVFP4 parameter tuples compiles as ONE
    graph (fullgraph=True: the ops trace through their fake kernels, no graph break) and its outputs equal eager's
    bit for bit, at a few-rows and a many-rows M;
  - the same calls, plus the gated and residual linears and the code readout, captured in a torch.cuda.graph and
    replayed after new inputs were copied into the captured buffers, equal eager on those inputs bit for bit, on two
    replays in a row.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import basal_b200
    return basal_b200


def _layers(b2, K=512, N=384, seed=0):
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(K, N, bias=True)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(N, generator=g) * 0.1)
    lin = lin.cuda()
    from basal_b200 import lean
    return (lean._params(b2.fp8block.BlockFP8Linear.of(lin)), lean._params(b2.int8block.Int8BlockLinear.of(lin)),
            lean._params(b2.nvfp4.NVFP4Linear.of(lin, 4.0)))


def test_compiled_layer_function_traces_as_one_graph(b2):
    from basal_b200 import lean
    p8, pi8, p4 = _layers(b2)

    def layer(x, p8, pi8, p4):
        return lean.linear(x, p8), lean.linear(x, pi8), lean.linear(x, p4)

    compiled = torch.compile(layer, fullgraph=True, dynamic=False)
    g = torch.Generator().manual_seed(1)
    for M in (16, 300):
        x = torch.randn(2, M, 512, generator=g).bfloat16().cuda()
        want = layer(x, p8, pi8, p4)
        got = compiled(x, p8, pi8, p4)
        for a, b in zip(got, want):
            assert a.shape == b.shape and a.dtype == b.dtype
            assert torch.equal(a, b)
    assert b2._lib.device_faults(0) == 0


def test_cuda_graph_capture_and_replay_on_new_inputs(b2):
    from basal_b200 import lean
    p8, pi8, p4 = _layers(b2, seed=2)
    K, N, I = 512, 384, 256
    g = torch.Generator().manual_seed(3)
    wg, sg = b2.fp8block.quantize((torch.randn(2 * I, K, generator=g) * 0.02).cuda())
    head = torch.nn.Linear(K, 1000, bias=False).to(torch.bfloat16).cuda()
    ro = b2.readout.CodeReadout(head, softcap=30.0)
    rows, idx, pad = ro.rows([[5, 9, 700], [1, 2], [999, 0, 3, 4]] * 5)

    def forward(x, r):
        y8 = lean.linear(x, p8)
        return (y8, lean.linear(x, pi8), lean.linear(x, p4), b2.fp8block.linear_glu(x, wg, sg, "silu"),
                b2.fp8block.FORMAT.linear_residual(x, p8[0], p8[1], None, r),
                ro.probs_of(ro.logits(x[:15].float(), rows), idx, pad))

    for M in (15, 1000):
        static_x = torch.randn(M, K, generator=g).bfloat16().cuda()
        static_r = torch.randn(M, N, generator=g).bfloat16().cuda()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):  # warm-up off the capturing stream, as torch recommends
                forward(static_x, static_r)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = forward(static_x, static_r)
        for _ in range(2):
            x = torch.randn(M, K, generator=g).bfloat16().cuda()
            r = torch.randn(M, N, generator=g).bfloat16().cuda()
            static_x.copy_(x)
            static_r.copy_(r)
            graph.replay()
            torch.cuda.synchronize()
            want = forward(x, r)
            for i, (a, b) in enumerate(zip(outs, want)):
                assert torch.equal(a, b), (M, i)
        del graph
    assert b2._lib.device_faults(0) == 0
