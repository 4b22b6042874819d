#pragma once
#define LAMMPS_VERSION "mock"
