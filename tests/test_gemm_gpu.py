"""The tcgen05 GEMM and its epilogues against an fp64 product of the same bf16
operands (2e-2 relative for bf16 outputs, 1e-3 for fp32 outputs of bf16 data)."""
import pytest
import torch

from conftest import rel_err
from hclsm_b200.kernels.gemm import gemm_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(4096, 384, 384), (4096, 1536, 384), (4096, 384, 1536), (1856, 1152, 384),
                                   (1, 128, 64), (300, 256, 192)])
@pytest.mark.parametrize("epi", ["none", "relu", "resid"])
def test_gemm_epilogues(M, N, K, epi):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    bias = torch.randn(N, generator=g).cuda()
    resid = torch.randn(M, N, generator=g).cuda() if epi == "resid" else None
    of, ob = gemm_bf16(a, w, bias=bias, epilogue=epi, resid=resid, clamp=1.5 if epi == "resid" else 0.0,
                       out_f32=True, out_bf16=True)
    ref = a.double() @ w.double().T + bias.double()
    if epi == "relu":
        ref = ref.clamp_min(0)
    if epi == "resid":
        ref = (ref + resid.double()).clamp(-1.5, 1.5)
    assert rel_err(of.cpu().numpy(), ref.cpu().numpy()) < 1e-3
    assert rel_err(ob.float().cpu().numpy(), ref.cpu().numpy()) < 2e-2
