"""Numerical tolerances for the bf16 hot path.

The north-star bar is 2e-2 relative error on bf16 activations with fp32
accumulation. A tensor passes when
  * its relative Frobenius error ||got - ref|| / ||ref|| <= REL_FRO, and
  * every element satisfies |got - ref| <= RTOL * |ref| + ATOL_RMS * rms(ref)
    (the rms term covers elements near zero, where one bf16 ulp of a
    differently ordered fp32 sum is large relative to the element).
"""
import torch

RTOL = 2e-2
REL_FRO = 2e-2
ATOL_RMS = 2e-2
# Hidden states after several layers: bf16 residual adds of operands up to
# ~4x the row rms cancel, so one ulp of an operand can be several % of rms.
ATOL_RMS_MULTILAYER = 5e-2


def assert_close(got: torch.Tensor, ref: torch.Tensor, what: str = "", rtol: float = RTOL,
                 rel_fro: float = REL_FRO, atol_rms: float = ATOL_RMS) -> None:
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert g.shape == r.shape, f"{what}: shape {tuple(g.shape)} != {tuple(r.shape)}"
    if r.numel() == 0:
        return
    d = (g - r).abs()
    rms = r.pow(2).mean().sqrt().item()
    fro = (d.pow(2).sum().sqrt() / max(r.pow(2).sum().sqrt().item(), 1e-30)).item()
    assert torch.isfinite(g).all(), f"{what}: non-finite values"
    assert fro <= rel_fro, f"{what}: relative Frobenius error {fro:.3e} > {rel_fro}"
    bound = rtol * r.abs() + atol_rms * rms
    bad = d > bound
    if bad.any():
        i = int(bad.flatten().nonzero()[0])
        raise AssertionError(
            f"{what}: {int(bad.sum())} elements out of tolerance (rel Frobenius {fro:.3e}, "
            f"max |diff|/rms {d.max().item() / max(rms, 1e-30):.3e}); first at flat index {i}: "
            f"got {g.flatten()[i].item():.6g} ref {r.flatten()[i].item():.6g}")
