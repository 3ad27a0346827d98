"""The bf16 batched transpose (gsq_transpose_bf16): 16-byte vector and single-element paths,
ragged edges, and the causal skip (only the transposes of tiles above the 128-block diagonal are
left unwritten)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _T(x, rows, cols, ld_in, bs_in, out, ld_out, bs_out, batch, skip=0):
    from gsq_rco_mlx_b200 import _lib
    _lib.call("gsq_transpose_bf16", _lib.ptr(x), rows, cols, ld_in, bs_in, _lib.ptr(out), ld_out,
              bs_out, batch, skip, _lib.stream_ptr())
    torch.cuda.synchronize()


@pytest.mark.parametrize("rows,cols,ld_in,ld_out", [(256, 192, 192, 256), (130, 77, 80, 136),
                                                    (100, 70, 73, 101)])
def test_transpose_matches_torch(rows, cols, ld_in, ld_out):
    g = torch.Generator(device=DEV).manual_seed(0)
    B = 3
    x = torch.randn(B, rows, ld_in, device=DEV, generator=g).bfloat16()
    out = torch.zeros(B, cols, ld_out, device=DEV, dtype=torch.bfloat16)
    _T(x, rows, cols, ld_in, rows * ld_in, out, ld_out, cols * ld_out, B)
    assert torch.equal(out[:, :, :rows], x[:, :, :cols].transpose(1, 2))


def test_transpose_causal_skip():
    g = torch.Generator(device=DEV).manual_seed(1)
    T, B = 320, 2
    x = torch.tril(torch.randn(B, T, T, device=DEV, generator=g)).bfloat16()
    out = torch.full((B, T, T), 7.0, device=DEV, dtype=torch.bfloat16)
    _T(x, T, T, T, T * T, out, T, T * T, B, skip=1)
    r = torch.arange(T, device=DEV)
    read = (r[:, None] >> 7) <= (r[None, :] >> 7)       # out[c][r] with (c >> 7) <= (r >> 7)
    ref = x.transpose(1, 2)
    assert torch.equal(out[:, read], ref[:, read])
    assert bool((out[:, ~read] == 7.0).all())              # never written
