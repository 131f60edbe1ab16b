"""Host-side shape rules shared by the torch ops and the numpy front-end
(no GPU): accepted layouts and the ValueError for each misfit."""

import pytest

from armhackathon_b200.layout import m1_layout


def test_accepts_plain_and_grouped_bc():
    lay = m1_layout((2, 8, 5), (2, 8, 5), (8, 4), (2, 4, 5), (2, 4, 5), D=(8,), z=(2, 8, 5),
                    delta_bias=(8,), initial_state=(2, 8, 4))
    assert (lay.batch, lay.dim, lay.length, lay.state, lay.groups) == (2, 8, 5, 4, 1)
    assert lay.bc_shape == (2, 1, 4, 5)
    assert m1_layout((2, 8, 5), (2, 8, 5), (8, 4), (2, 2, 4, 5), (2, 2, 4, 5)).groups == 2


@pytest.mark.parametrize("kw,msg", [
    (dict(delta=(2, 8, 6)), "delta"), (dict(A=(7, 4)), "A must"), (dict(B=(2, 3, 5)), "B must"),
    (dict(C=(2, 2, 4, 5)), "disagree"), (dict(B=(2, 3, 4, 5), C=(2, 3, 4, 5)), "divide"),
    (dict(D=(7,)), "D must"), (dict(z=(2, 8, 4)), "z must"), (dict(delta_bias=(9,)), "delta_bias"),
    (dict(initial_state=(2, 8, 3)), "initial_state"), (dict(u=(8, 5)), "u must"),
])
def test_rejects_misfits(kw, msg):
    args = dict(u=(2, 8, 5), delta=(2, 8, 5), A=(8, 4), B=(2, 4, 5), C=(2, 4, 5))
    args.update(kw)
    with pytest.raises(ValueError, match=msg):
        m1_layout(**args)
