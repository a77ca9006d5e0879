"""Host-side mirrors of the reference's utils/ ops, backed by libvhope.so."""
