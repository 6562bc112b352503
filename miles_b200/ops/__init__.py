"""Python entry points of the sm_100a kernel library."""
from miles_b200.ops._lib import check_device_error, native_available  # noqa: F401
