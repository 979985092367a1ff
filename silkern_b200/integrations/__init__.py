"""Runtime integrations; each submodule targets one upstream call site."""
