"""GPU checks of the library boundary: the loaded kernels are sm_100a code."""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


def test_loaded_kernels_are_sm100(ctx):
    import realm_b200 as rb
    v = C.c_int32()
    assert rb.lib().rb_kernel_binary_version(ctx.handle, C.byref(v)) == 0, rb.last_error()
    assert v.value == 100, v.value
