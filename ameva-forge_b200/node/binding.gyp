{
  "targets": [
    {
      "target_name": "forge_b200",
      "sources": ["forge_b200_addon.cc"],
      "include_dirs": ["../../include"],
      "cflags_cc": ["-std=c++17", "-O2"],
      "libraries": ["-L<(module_root_dir)/../forge_b200/_lib", "-lforge_b200",
                    "-Wl,-rpath,<(module_root_dir)/../forge_b200/_lib"]
    }
  ]
}
