"""B200-native differentiable Gaussian-splat renderer and L1/SSIM loss."""
