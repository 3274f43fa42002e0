"""Oracle package: CPU restatement of the reference's linear-layer arithmetic
plus bindings to the reference's own CPU code built from source.

TEST INFRASTRUCTURE ONLY -- see oracle/oracle.py."""
