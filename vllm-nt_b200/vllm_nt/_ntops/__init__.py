"""Plugin internals: config, router, hooks (patching), adapters (oot_support), torch
wrappers (torch/) and the ctypes view of the C ABI (capi)."""
