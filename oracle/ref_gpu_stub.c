/* Stub device entry points for building the reference engine as a CPU-only binary.
 * TEST INFRASTRUCTURE ONLY: every call reports failure, so the engine can run
 * only with its cpu backend (src/minimind.h:16-22 declares these symbols). */
int gpu_init(const void *file, unsigned bytes) { (void)file; (void)bytes; return 1; }
int gpu_forward(float *l, int t, int p, int pr, int r) { (void)l; (void)t; (void)p; (void)pr; (void)r; return 1; }
int gpu_finish(void) { return 1; }
int gpu_head_init(const void *file) { (void)file; return 1; }
int gpu_head_start(const float *x, int rows) { (void)x; (void)rows; return 1; }
int gpu_head_finish(float *l, int rows, int r) { (void)l; (void)rows; (void)r; return 1; }
int gpu_collect(float *l, const int *h, int c, float p, int k, int rows)
{ (void)l; (void)h; (void)c; (void)p; (void)k; (void)rows; return 1; }
