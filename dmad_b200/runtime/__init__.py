"""Runtime services: config, checkpoint / resume, logging and metrics, watchdog, callbacks, profiling."""
