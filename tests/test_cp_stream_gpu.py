"""Context-parallel attention with keys and values read in place from their
owners (the streaming form), on ONE GPU: every "owner" is a separate compact
[B, Tl, 2C] buffer on this device, so the per-owner TMA maps, the owner/row
arithmetic of both splits and the publish-word waits run without any peer
memory or cross-process wait. The streamed kernels load the same blocks in
the same order as the kernels given the gathered (natural-order) keys and
values, so outputs, LSE and gradients must match bit for bit; a publish word
that never reaches the epoch must end the launch with ERR_TIMEOUT_PEER and
leave the context usable.

These kernels have not yet run on a GPU. Until they have, the tests run only
when G2B_CP_STREAM_GPU=1 is set, so that a default GPU-tier run never
executes them first."""

import os

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("G2B_CP_STREAM_GPU") != "1",
                                 reason="streamed-KV kernels: set G2B_CP_STREAM_GPU=1 to run")]

from gpt2_harness_b200.ops import native as N  # noqa: E402

ERR_TIMEOUT_PEER = 1 << 3


def dev():
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _errors_clean():
    torch.cuda.set_device(0)
    N.error_word().zero_()
    yield
    torch.cuda.synchronize()


def _owner_of(k0: int, span: int, world: int, zigzag: bool):
    c = k0 // span
    if not zigzag:
        return c, 0
    return (c, 0) if c < world else (2 * world - 1 - c, span)


def _setup(world: int, zigzag: bool, B=2, H=4, Tl=256, epoch=5):
    C = H * 64
    T = world * Tl
    g = torch.Generator(device="cpu").manual_seed(world * 10 + int(zigzag))
    owners = [torch.randn(B, Tl, 2 * C, generator=g).bfloat16().to(dev()) for _ in range(world)]
    natural = torch.empty(B, T, 2 * C, dtype=torch.bfloat16, device=dev())
    span = Tl // 2 if zigzag else Tl
    for k0 in range(0, T, span):
        q, r0 = _owner_of(k0, span, world, zigzag)
        natural[:, k0:k0 + span] = owners[q][:, r0:r0 + span]
    flags = torch.full((16,), epoch, dtype=torch.int32, device=dev())
    peers = {"bases": [o.data_ptr() for o in owners], "sb": Tl * 2 * C, "st": 2 * C, "v_off": C, "Tl": Tl,
             "zigzag": int(zigzag), "flags": flags.data_ptr(), "epoch": epoch}
    return C, T, owners, natural.view(B * T, 2 * C), flags, peers


def _query_spans(rank: int, world: int, Tl: int, zigzag: bool):
    """(local row offset, queries, natural position of the first, keys seen)."""
    if not zigzag:
        return [(0, Tl, rank * Tl, (rank + 1) * Tl)]
    h = Tl // 2
    return [(half * h, h, k * h, (k + 1) * h) for half, k in enumerate((rank, 2 * world - 1 - rank))]


@pytest.mark.parametrize("world,zigzag", [(2, False), (2, True), (4, True), (8, True)])
def test_streamed_attention_matches_gathered(world, zigzag):
    B, H, Tl = 2, 4, 256
    C, T, owners, kvn, flags, peers = _setup(world, zigzag, B, H, Tl)
    for rank in (0, world - 1):
        q = torch.randn(B * Tl, C, device=dev()).bfloat16()
        dy = torch.randn(B * Tl, C, device=dev()).bfloat16()
        res = {}
        for mode in ("gathered", "streamed"):
            o = torch.zeros(B * Tl, C, dtype=torch.bfloat16, device=dev())
            lse = torch.zeros(2, B, H, Tl, device=dev())
            delta = torch.zeros(2, B, H, Tl, device=dev())
            dq = torch.zeros(B * Tl, C, dtype=torch.bfloat16, device=dev())
            dkv = torch.zeros(2, B * T, 2 * C, dtype=torch.bfloat16, device=dev())
            for i, (r0, n, q0, Tk) in enumerate(_query_spans(rank, world, Tl, zigzag)):
                L = lse[i].view(-1)[: B * H * n].view(B, H, n)
                D = delta[i].view(-1)[: B * H * n].view(B, H, n)
                if mode == "gathered":
                    N.attention_fwd(q[r0:], kvn[:, :C], kvn[:, C:], o[r0:], L, B, H, n, Tk=Tk, q_offset=q0,
                                    kv_rows=T, q_rows=Tl)
                    N.attention_bwd(q[r0:], kvn[:, :C], kvn[:, C:], o[r0:], dy[r0:], dq[r0:], dkv[i][:, :C],
                                    dkv[i][:, C:], L, D, B, H, n, Tk=Tk, q_offset=q0, kv_rows=T, q_rows=Tl)
                else:
                    N.attention_fwd_peers(q[r0:], o[r0:], L, B, H, n, Tk, q0, peers, q_rows=Tl)
                    N.attention_bwd_peers(q[r0:], o[r0:], dy[r0:], dq[r0:], dkv[i][:, :C], dkv[i][:, C:], L, D,
                                          B, H, n, Tk, q0, peers, kv_rows=T, q_rows=Tl)
            torch.cuda.synchronize()
            N.check_errors()
            res[mode] = (o, lse, dq, dkv)
        for name, a, b in zip(("o", "lse", "dq", "dkv"), res["gathered"], res["streamed"]):
            assert torch.equal(a, b), (name, rank, (a.float() - b.float()).abs().max().item())


def test_unpublished_owner_times_out_and_context_survives():
    """An owner whose publish word never reaches the epoch: the producer's
    bounded wait gives up, the launch records ERR_TIMEOUT_PEER and returns,
    and the context still runs work."""
    world, B, H, Tl = 2, 1, 2, 256
    C, T, owners, kvn, flags, peers = _setup(world, False, B, H, Tl)
    flags[1] = 4  # rank 1 never published epoch 5
    q = torch.randn(B * Tl, C, device=dev()).bfloat16()
    o = torch.zeros(B * Tl, C, dtype=torch.bfloat16, device=dev())
    lse = torch.zeros(B, H, Tl, device=dev())
    N.attention_fwd_peers(q, o, lse, B, H, Tl, 2 * Tl, Tl, peers)  # rank 1's queries see rank 1's keys
    torch.cuda.synchronize()
    err = int(N.error_word().item())
    assert err & ERR_TIMEOUT_PEER, err
    N.error_word().zero_()
    x = torch.ones(4, device=dev())
    assert x.sum().item() == 4
