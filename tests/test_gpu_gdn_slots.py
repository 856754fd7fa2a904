"""GDN state commit as a slot index (tlx_gdn_slots_init / tlx_acceptsel11k_flip)
against the copy it replaces (tlx_acceptsel11k, checked bit-exact against the
reference kernel in test_gpu_refkernels.py).

Both forms run the same sequence of steps on their own copies of the buffers: every
step writes new draft states for all eleven positions (the copy form at the
reference's fixed addresses, the index form at the addresses its table names), then
accepts a position m.  After each accept the live state read through the table must
equal the copy form's live slot bit for bit, and the table must stay a permutation of
the physical buffers (rec draft 4 aliasing the live state, as in the reference
layout)."""
import numpy as np
import pytest
import torch

from thunderllamax_b200 import ops

pytestmark = pytest.mark.gpu

NB, REC, CONV = 3, 64, 32


def _buffers(rng):
    f = lambda n: torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()  # noqa: E731
    return {"rec4": f(NB * 5 * REC), "conv4": f(NB * 5 * CONV),
            "conv_x": [f(NB * CONV) for _ in range(7)], "rec_x": [f(NB * REC) for _ in range(6)]}


def _clone(bufs):
    return {"rec4": bufs["rec4"].clone(), "conv4": bufs["conv4"].clone(),
            "conv_x": [t.clone() for t in bufs["conv_x"]], "rec_x": [t.clone() for t in bufs["rec_x"]]}


def _fixed_view(bufs, b, kind, s):
    """The reference's fixed address of draft s (0..10) or the live state (11)."""
    if kind == 0:
        if s == 11 or s <= 4:
            slot = 4 if s == 11 else s
            return bufs["rec4"][(b * 5 + slot) * REC:(b * 5 + slot + 1) * REC]
        return bufs["rec_x"][s - 5][b * REC:(b + 1) * REC]
    if s == 11 or s <= 3:
        slot = 4 if s == 11 else s
        return bufs["conv4"][(b * 5 + slot) * CONV:(b * 5 + slot + 1) * CONV]
    return bufs["conv_x"][s - 4][b * CONV:(b + 1) * CONV]


def _resolver(bufs):
    """device address -> view of the buffer element range it starts"""
    table = {}
    for kind, elems in ((0, REC), (1, CONV)):
        for b in range(NB):
            for s in range(12):
                v = _fixed_view(bufs, b, kind, s)
                table[v.data_ptr()] = v
    return table


def test_flip_equals_copy_over_steps():
    ops.require_device()
    rng = np.random.default_rng(11)
    cp = _buffers(rng)
    ix = _clone(cp)
    slots = ops.GdnSlots(ix["rec4"], ix["conv4"], ix["conv_x"], ix["rec_x"], NB, REC, CONV)
    where = _resolver(ix)
    m_slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    seen = set()
    for step, m in enumerate([7, 0, 4, 10, 3, 5, 9, 1, 6, 2, 8, 4, 11, -1, 10]):
        tab = slots.entries()
        # the next step's draft states, the same values in both forms
        for b in range(NB):
            for kind, elems in ((0, REC), (1, CONV)):
                for s in range(11):
                    val = torch.from_numpy(rng.standard_normal(elems).astype(np.float32)).cuda()
                    _fixed_view(cp, b, kind, s).copy_(val)
                    where[int(tab[b, kind, s])].copy_(val)
        m_slot.fill_(m)
        ops.acceptsel11k(cp["rec4"], cp["conv4"], m_slot, cp["conv_x"], cp["rec_x"], NB, REC, CONV)
        slots.flip(m_slot)
        torch.cuda.synchronize()
        tab = slots.entries()
        for b in range(NB):
            for kind in (0, 1):
                live = where[int(tab[b, kind, 11])]
                assert torch.equal(live, _fixed_view(cp, b, kind, 11)), (step, m, b, kind)
            rec, conv = [int(a) for a in tab[b, 0]], [int(a) for a in tab[b, 1]]
            assert rec[4] == rec[11] and len(set(rec[:11])) == 11, (step, b)
            assert len(set(conv)) == 12, (step, b)
            assert set(rec) <= set(where) and set(conv) <= set(where)
        seen.add(m)
    assert {0, 4, 10, 11, -1} <= seen


def test_flip_rejects_bad_arguments():
    ops.require_device()
    from thunderllamax_b200 import _lib
    L = _lib.lib()
    assert L.tlx_gdn_slots_bytes(48) == 48 * 2 * 12 * 8
    assert L.tlx_gdn_slots_bytes(0) == 0
    assert L.tlx_acceptsel11k_flip(None, None, 48, None) < 0
    t = torch.zeros(8, dtype=torch.int64, device="cuda")
    m = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.tlx_acceptsel11k_flip(ctypes_ptr(t), ctypes_ptr(m), 0, None) < 0


def ctypes_ptr(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())
