"""GPU tests of the expert-parallel pieces on one device: the layout kernel
against its host restatement, and N ranks emulated on one GPU through the real
kernels (pack, layout, grouped FFN on the receive layout, unpermute) with the
AllToAllv replaced by indexing.  Each output row of the FFN depends only on
its own input row and expert, so the emulated EP layer must be bit-identical
to the single-GPU layer."""
import numpy as np
import pytest
import torch

import ep
import moe_b200 as mb
import routing

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,E", [(1, 8), (2, 8), (4, 10), (8, 60), (8, 8), (3, 64)])
def test_ep_layout_kernel_matches_reference(cuda, N, E):
    rng = np.random.default_rng(N * 100 + E)
    counts = rng.integers(0, 300, size=(N, E)).astype(np.int32)
    counts[0, 0] = 0
    b = ep.expert_ranges(E, N)
    dc = torch.from_numpy(counts).cuda()
    for r in range(N):
        ss, se, send, recv = mb.ep_layout(dc, r, b)
        rs, re_, rsend, rrecv = ep.layout_reference(counts.tolist(), r, b)
        assert ss.tolist() == rs
        L = b[r + 1] - b[r]
        assert se[: N * L].tolist() == re_
        assert send.tolist() == rsend
        assert recv.tolist() == rrecv


def test_ep_layout_rejects_bad_bounds(cuda):
    dc = torch.zeros((2, 4), dtype=torch.int32, device="cuda")
    with pytest.raises(mb.MoEB200Error):
        mb.ep_layout(dc, 0, [0, 3, 3])  # does not end at E
    with pytest.raises(mb.MoEB200Error):
        mb.ep_layout(dc, 2, [0, 2, 4])  # rank out of range


def test_emulated_ep_layer_bit_identical_to_single_gpu(cuda):
    N, Tr, K, E, d, I = 4, 1024, 4, 16, 256, 128
    dtype = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    wgu = (torch.randn((E, 2 * I, d), generator=g, device="cuda") * 0.02).to(dtype)
    wdn = (torch.randn((E, d, I), generator=g, device="cuda") * 0.02).to(dtype)
    b = ep.expert_ranges(E, N)
    packs, xs, ws = [], [], []
    for r in range(N):
        asgn, wts = routing.gen_routing(Tr, K, E, "zipf", seed=r)
        x = routing.gen_rows(Tr, d, "bfloat16", seed=r, device="cuda")
        w = torch.from_numpy(wts).cuda()
        packs.append(mb.pack(x, torch.from_numpy(asgn).cuda(), w, E))
        xs.append(x)
        ws.append(w)
    all_counts = torch.stack([p.expert_count for p in packs])
    # emulated dispatch: receiver r takes sender g's rows of r's experts
    recv_bufs, layouts = [], []
    for r in range(N):
        lay = mb.ep_layout(all_counts, r, b)
        parts = [packs[g].packed[packs[g].expert_start[b[r]]:packs[g].expert_start[b[r + 1]]] for g in range(N)]
        recv_bufs.append(torch.cat(parts))
        layouts.append(lay)
        assert recv_bufs[r].shape[0] == int(lay[3].sum())
    # expert FFN on every receiver with its local weights
    ys = []
    for r in range(N):
        ss, se = layouts[r][0], layouts[r][1]
        _, y = mb.grouped_swiglu(recv_bufs[r], ss, wgu[b[r]:b[r + 1]].contiguous(),
                                 wdn[b[r]:b[r + 1]].contiguous(), seg_expert=se)
        ys.append(y)
    assert mb.device_status() == 0
    # emulated combine + unpermute, compared with the single-GPU layer per sender
    for g in range(N):
        back = torch.empty_like(packs[g].packed)
        for r in range(N):
            lo = int(packs[g].expert_start[b[r]])
            hi = int(packs[g].expert_start[b[r + 1]])
            off = int(layouts[r][3][:g].sum())
            back[lo:hi] = ys[r][off:off + (hi - lo)]
        out_ep = mb.unpermute(back, packs[g].packed_weights, packs[g].slot_pos, Tr, K)
        _, y1 = mb.grouped_swiglu(packs[g].packed, packs[g].expert_start, wgu, wdn)
        out_1 = mb.unpermute(y1, packs[g].packed_weights, packs[g].slot_pos, Tr, K)
        assert torch.equal(out_ep.view(torch.int16), out_1.view(torch.int16))
