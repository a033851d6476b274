"""Mirror of jax_2dgs (2D Gaussian surfel splatting) on libgsb200."""
