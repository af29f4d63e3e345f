"""Host-side core: configs, mu_clamp, paged cache bookkeeping, scheduler."""
