"""sm_100a kernel wrappers: codecs (``ops.codecs``) and the device ``.nz``
trajectory pipeline (``ops.trajectory``)."""
