"""SGLang integration of the packed-state pool (hooks mirror stepquant/sglang/*).

Importing this package does not import SGLang; ``plugin.register`` does, and
only when ``STEPQUANT_PLAN`` or ``STEPQUANT_STATE_FORMAT`` is set.
"""
