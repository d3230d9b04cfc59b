"""Host-side layout of the peer-memory expert-parallel dispatch: every assignment of every source rank lands on
a distinct row inside its expert's segment on the owning rank, rows of lower source ranks first."""
import numpy as np


def test_ep_host_layout_is_a_partition():
    from elasticmegatron_b200.ops.ep_comm import SEG_ALIGN, host_layout

    rng = np.random.default_rng(0)
    for ep, e_loc in ((2, 4), (4, 2), (8, 1), (4, 3)):
        E = ep * e_loc
        ac = rng.integers(0, 300, size=(ep, E))
        ac[0, 0] = 0
        rows = {d: set() for d in range(ep)}
        for src in range(ep):
            _, _, base, _, _, _ = host_layout(ac, src, e_loc)
            for eg in range(E):
                d, e = divmod(eg, e_loc)
                seg_d, tot_d, _, tiles_d, cap_d, _ = host_layout(ac, d, e_loc)
                for j in range(ac[src, eg]):
                    r = base[eg] + j
                    assert seg_d[e] <= r < seg_d[e] + tot_d[e], (src, eg, j)
                    assert tiles_d[r // SEG_ALIGN] == e
                    assert r not in rows[d]
                    rows[d].add(r)
                if src > 0:  # lower source ranks come first inside a segment
                    assert base[eg] == seg_d[e] + ac[:src, eg].sum()
        for d in range(ep):
            seg_d, tot_d, _, _, cap_d, cap_max = host_layout(ac, d, e_loc)
            assert len(rows[d]) == tot_d.sum() and cap_d % SEG_ALIGN == 0 and cap_d <= cap_max
            assert all((seg_d[e + 1] - seg_d[e]) % SEG_ALIGN == 0 for e in range(e_loc))
