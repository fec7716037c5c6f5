"""CUDA-graph capture of the hot-path launches: a decode sequence of grouped
W4A16 GEMV launches (programmatic dependent launch between them), the tcgen05
W4A16 and FP8 GEMMs, and the MLP block, captured once with torch.cuda.graph
and replayed with new activations copied into the captured input buffers.
Every replay must equal an eager run of the same launches bit for bit (same
kernels, same inputs), and no device-side wait may give up."""
import pytest
import torch

import kc_lib
import kernel_craft_torch_ops as ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_timeouts(cuda):
    yield
    assert kc_lib.lib().kc_get_device_status() == kc_lib.KC_OK


def _w4(g, N, K, gs=128):
    p = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    s = (torch.rand(N, K // gs, device="cuda", generator=g) * 0.018 + 0.002).half()
    return p, s


def _replay_matches_eager(run, inputs, outputs_of, new_inputs):
    """Capture run() once, then for each set of new input values: copy them
    into the captured inputs, replay, and compare with an eager run()."""
    run()                                    # warm-up outside capture (attributes, maps)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = run()
    for values in new_inputs:
        for dst, src in zip(inputs, values):
            dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize()
        got = [o.clone() for o in outputs_of(outs)]
        want = outputs_of(run())
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            assert torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                               b.view(torch.int16) if b.dtype == torch.bfloat16 else b)


def test_decode_gemv_sequence_graph(cuda):
    g = torch.Generator(device="cuda").manual_seed(1)
    shapes = [(4096, 1536), (4096, 512), (1024, 2752), (1408, 512)]      # (K, N)
    layers = []
    for _ in range(4):
        probs = []
        for K, N in shapes:
            p, s = _w4(g, N, K)
            probs.append((p, s, torch.randn(1, K, device="cuda", generator=g).bfloat16()))
        layers.append(probs)
    xs = [x for probs in layers for _, _, x in probs]

    def run():
        return [ops.w4a16_gemv_grouped(probs, 128) for probs in layers]

    new = [[torch.randn(x.shape, device="cuda", generator=g).bfloat16() for x in xs] for _ in range(3)]
    _replay_matches_eager(run, xs, lambda outs: [y for ys in outs for y in ys], new)


def test_gemms_graph(cuda):
    g = torch.Generator(device="cuda").manual_seed(2)
    M, N, K = 256, 512, 1024
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    p, s = _w4(g, N, K)
    a = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    qw, sw = ops.fp8_quantize_per_channel(w)

    def run():
        qa, sa = ops.fp8_quantize(a, per_token=True)
        return (ops.w4a16_gemm(x, p, s, 128, activation="gelu_quick"),
                ops.fp8_gemm(qa, sa, qw, sw, out_dtype=torch.float32))

    new = [(torch.randn(x.shape, device="cuda", generator=g).bfloat16(),
            torch.randn(a.shape, device="cuda", generator=g)) for _ in range(2)]
    _replay_matches_eager(run, [x, a], lambda outs: list(outs), new)


def test_mlp_block_graph(cuda):
    import tp
    g = torch.Generator(device="cuda").manual_seed(3)
    M, H, I = 128, 512, 1024
    x = torch.randn(M, H, device="cuda", generator=g).bfloat16()
    w1p, w1s = _w4(g, I, H)
    w2p, w2s = _w4(g, H, I)
    blk = tp.MLPBlockW4A16(M, H, I, 128)

    def run():
        return blk(x, w1p, w1s, w2p, w2s)

    new = [(torch.randn(x.shape, device="cuda", generator=g).bfloat16(),) for _ in range(2)]
    _replay_matches_eager(run, [x], lambda y: [y], new)
