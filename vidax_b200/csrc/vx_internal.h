// Library-internal helpers shared by the translation units of libvidax_cuda.so.
#pragma once

// Records `msg` as the calling thread's last error (vx_last_error) and
// returns `code`.
int vx_internal_fail(int code, const char* msg);

// Device address of the current device's status word (the one
// vx_device_status reads), looked up once per device.
int vx_internal_status_word(int** out);
