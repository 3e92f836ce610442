{
  "targets": [
    {
      "target_name": "nsattn_addon",
      "sources": ["nsattn_addon.c"],
      "include_dirs": ["../../include"],
      "libraries": ["-L<(module_root_dir)/..", "-lnsattn", "-Wl,-rpath,<(module_root_dir)/.."],
      "cflags": ["-std=c11", "-Wall"]
    }
  ]
}
