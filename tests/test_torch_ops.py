"""The torch.library operators: schemas and fake (shape) implementations on the
CPU; on a GPU, the ops give the same results as the direct calls."""
import pytest
import torch


def test_ops_registered_with_schemas(nv):
    import nvfp4_b200.torch_ops  # noqa: F401
    g = torch.ops.nvfp4_b200.gemm
    q = torch.ops.nvfp4_b200.quantize
    assert "Tensor a" in str(g.default._schema) and "float alpha" in str(g.default._schema)
    assert "Tensor global_scale" in str(q.default._schema)


def test_fake_shapes_without_a_gpu(nv):
    import nvfp4_b200.torch_ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        a = torch.empty(300, 256, dtype=torch.uint8)
        b = torch.empty(1000, 256, dtype=torch.uint8)
        sfa = torch.empty(384 * 32, dtype=torch.uint8)
        sfb = torch.empty(1024 * 32, dtype=torch.uint8)
        d = torch.ops.nvfp4_b200.gemm(a, sfa, b, sfb, 1.0)
        assert d.shape == (300, 1000) and d.dtype == torch.bfloat16
        d16 = torch.ops.nvfp4_b200.gemm(a, sfa, b, sfb, 1.0, True)
        assert d16.dtype == torch.float16
        x = torch.empty(300, 512, dtype=torch.bfloat16)
        qq, sf = torch.ops.nvfp4_b200.quantize(x, torch.empty(1))
        assert qq.shape == (300, 256) and sf.shape == (384 * 32,)


@pytest.mark.gpu
def test_ops_match_direct_calls(nv, cuda_dev):
    import nvfp4_b200.torch_ops  # noqa: F401
    x = torch.randn(512, 1024, device=cuda_dev).to(torch.bfloat16)
    w = (torch.randn(768, 1024, device=cuda_dev) * 0.02).to(torch.bfloat16)
    _, gx = nv.global_scale(x)
    _, gw = nv.global_scale(w)
    q1, s1 = torch.ops.nvfp4_b200.quantize(x, gx)
    q2, s2 = nv.quantize(x, gx)
    wq, ws = nv.quantize(w, gw)
    assert torch.equal(q1, q2) and torch.equal(s1, s2)
    d1 = torch.ops.nvfp4_b200.gemm(q1, s1, wq, ws, 0.5)
    d2 = nv.gemm(q2, s2, wq, ws, 0.5)
    torch.cuda.synchronize()
    assert torch.equal(d1, d2)
