"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the moebius-cpu engine kernels."""
