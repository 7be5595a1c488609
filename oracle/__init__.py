"""ORACLE — test infrastructure only (tests/, __graft_entry__.smoke(), bench.py's CPU baseline).

``oracle.semantics`` restates the reference's residual and apply semantics in NumPy;
``oracle.stream`` loads the plain-C decoder of the stream format (``stream_oracle.c``).
Nothing in ``warpshift_b200`` imports this package.
"""
