{
  "targets": [
    {
      "target_name": "tabnet_b200",
      "sources": ["tabnet_b200.c"],
      "include_dirs": ["../include"],
      "libraries": ["-L<(module_root_dir)/../ce-tabnet_b200", "-ltabnet_stage",
                    "-Wl,-rpath,<(module_root_dir)/../ce-tabnet_b200"],
      "cflags_c": ["-std=c11", "-O2", "-Wall"]
    }
  ]
}
