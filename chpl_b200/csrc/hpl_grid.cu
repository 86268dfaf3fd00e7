// Multi-GPU (P x Q) HPL driver.
