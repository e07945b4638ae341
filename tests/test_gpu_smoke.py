"""The round-end smoke check (``__graft_entry__.smoke``) runs inside the GPU suite too, so a change
that breaks it shows up with the other GPU tests."""

import pytest

pytestmark = pytest.mark.gpu


def test_smoke():
    import __graft_entry__

    __graft_entry__.smoke()
